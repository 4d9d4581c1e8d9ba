"""EnCodec (Meta's neural audio codec, 24 kHz mono / 48 kHz stereo): a SEANet
convolutional encoder / decoder with an LSTM, and a residual vector quantiser
with Euclidean codebooks whose number of stages follows the target bandwidth.

    conv(x)   pad (causal: all on the left; else split, the extra right padding
              making the strided windows cover the signal), zero or reflected,
              then conv; time_group_norm models add GroupNorm(1 group) after it
    resblock  shortcut(x) + conv1x1(elu(conv_k(elu(x), dilation d)))  (hidden = dim / compress)
    encoder   conv(C -> F, k7) -> per ratio r (reversed): resblocks, elu, conv(k 2r, stride r), channels x2
              -> y + LSTM(y) -> elu -> conv(-> hidden, k7)
    decoder   conv(hidden -> F 2^n, k7) -> y + LSTM(y) -> per ratio: elu, convT(k 2r, stride r) trimmed
              (causal: right side by trim_right_ratio), resblocks -> elu -> conv(-> C, k7)
    RVQ       n_q = floor(bandwidth * 1000 / (frame_rate * log2(codebook_size))) stages,
              code = argmin ||r - e||^2, r -= e[code]
    chunking  (48 kHz) chunks of ``chunk_length_s`` with stride (1 - overlap), per-chunk RMS
              normalisation (the scale travels with the codes), triangular overlap-add on decode

Every convolution and the LSTM run on the shared codec blocks
(``models/codec_common.py``): ELU, padding and dilation fused into the GEMM
operand by ``act_im2col``, skip inputs added in the GEMM epilogue, transposed
convs as GEMM + ``convt_fold``, LSTM gates accumulated by ``linear_acc`` and
applied by ``lstm_cell``. The quantiser's distance products stay in fp32 torch.

Checkpoint names: transformers' EncodecModel (``encoder.layers.N...``,
``quantizer.layers.i.codebook.embed``), weight norm in either serialisation.

Reference: the reference's rlx-encodec crate (facebook/encodec_24khz: SEANet
encoder / decoder, LSTM, RVQ with bandwidth-selected stages).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .codec_common import ConvRunner, GemmConv, fold_weight_norm


@dataclass
class EncodecConfig:
    target_bandwidths: list = field(default_factory=lambda: [1.5, 3.0, 6.0, 12.0, 24.0])
    sampling_rate: int = 24000
    audio_channels: int = 1
    normalize: bool = False
    chunk_length_s: float | None = None
    overlap: float | None = None
    hidden_size: int = 128
    num_filters: int = 32
    num_residual_layers: int = 1
    upsampling_ratios: list = field(default_factory=lambda: [8, 5, 4, 2])
    norm_type: str = "weight_norm"
    kernel_size: int = 7
    last_kernel_size: int = 7
    residual_kernel_size: int = 3
    dilation_growth_rate: int = 2
    use_causal_conv: bool = True
    pad_mode: str = "reflect"
    compress: int = 2
    num_lstm_layers: int = 2
    trim_right_ratio: float = 1.0
    codebook_size: int = 1024
    codebook_dim: int | None = None
    use_conv_shortcut: bool = True

    def __post_init__(self):
        if self.codebook_dim is None:
            self.codebook_dim = self.hidden_size

    @classmethod
    def from_dict(cls, d: dict) -> "EncodecConfig":
        names = {f for f in cls.__dataclass_fields__}
        return cls(**{k: v for k, v in d.items() if k in names})

    @property
    def hop_length(self) -> int:
        return math.prod(self.upsampling_ratios)

    @property
    def frame_rate(self) -> int:
        return math.ceil(self.sampling_rate / self.hop_length)

    @property
    def num_quantizers(self) -> int:
        return int(1000 * self.target_bandwidths[-1] // (self.frame_rate * math.ceil(math.log2(self.codebook_size))))

    @property
    def chunk_length(self) -> int | None:
        return None if self.chunk_length_s is None else int(self.chunk_length_s * self.sampling_rate)

    @property
    def chunk_stride(self) -> int | None:
        if self.chunk_length_s is None or self.overlap is None:
            return None
        return max(1, int((1.0 - self.overlap) * self.chunk_length))

    def quantizers_for(self, bandwidth: float | None) -> int:
        if bandwidth is None or bandwidth <= 0:
            return self.num_quantizers
        per_q = math.log2(self.codebook_size) * self.frame_rate
        return int(max(1, math.floor(bandwidth * 1000 / per_q)))


@dataclass
class _Layer:
    kind: str              # conv | convt | res | lstm | elu
    name: str
    k: int = 1
    stride: int = 1
    dil: int = 1
    res_dil: int = 1


def _layout(cfg: EncodecConfig, lstm: bool = True) -> tuple[list[_Layer], list[_Layer]]:
    """The transformers module lists (``encoder.layers.N`` / ``decoder.layers.N``);
    ``lstm=False``: the SEANet stacks without their LSTMs (Mimi)."""
    enc = [_Layer("conv", "encoder.layers.0", k=cfg.kernel_size)]
    for r in reversed(cfg.upsampling_ratios):
        for j in range(cfg.num_residual_layers):
            enc.append(_Layer("res", f"encoder.layers.{len(enc)}", res_dil=cfg.dilation_growth_rate ** j))
        enc.append(_Layer("elu", f"encoder.layers.{len(enc)}"))
        enc.append(_Layer("conv", f"encoder.layers.{len(enc)}", k=2 * r, stride=r))
    if lstm:
        enc.append(_Layer("lstm", f"encoder.layers.{len(enc)}"))
    enc.append(_Layer("elu", f"encoder.layers.{len(enc)}"))
    enc.append(_Layer("conv", f"encoder.layers.{len(enc)}", k=cfg.last_kernel_size))
    dec = [_Layer("conv", "decoder.layers.0", k=cfg.kernel_size)]
    if lstm:
        dec.append(_Layer("lstm", "decoder.layers.1"))
    for r in cfg.upsampling_ratios:
        dec.append(_Layer("elu", f"decoder.layers.{len(dec)}"))
        dec.append(_Layer("convt", f"decoder.layers.{len(dec)}", k=2 * r, stride=r))
        for j in range(cfg.num_residual_layers):
            dec.append(_Layer("res", f"decoder.layers.{len(dec)}", res_dil=cfg.dilation_growth_rate ** j))
    dec.append(_Layer("elu", f"decoder.layers.{len(dec)}"))
    dec.append(_Layer("conv", f"decoder.layers.{len(dec)}", k=cfg.last_kernel_size))
    return enc, dec


class EncodecModel:
    """``seanet_only``: load just the SEANet convolution stacks (no LSTM, no
    quantiser) for codecs built around them (Mimi)."""

    def __init__(self, cfg: EncodecConfig, weights, device="cpu", seanet_only: bool = False):
        self.cfg = cfg
        self.run = ConvRunner(device)
        self.device, self.dtype = self.run.device, self.run.dtype
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        keys = [k for k in weights.keys() if not seanet_only or k.startswith(("encoder.layers.", "decoder.layers."))]
        w = fold_weight_norm({k: get(k) for k in keys})
        dt, dev = self.dtype, self.device
        self.convs: dict[str, GemmConv] = {}
        self.norms: dict[str, tuple] = {}
        self.enc, self.dec = _layout(cfg, lstm=not seanet_only)
        transposed = {L.name for L in self.dec if L.kind == "convt"}
        for n, t in w.items():
            if n.endswith(".conv.weight"):
                base = n[:-len(".conv.weight")]
                self.convs[base] = GemmConv(t, w.get(base + ".conv.bias"), base in transposed, dt, dev)
                if base + ".norm.weight" in w:
                    self.norms[base] = (w[base + ".norm.weight"].to(dev), w[base + ".norm.bias"].to(dev))
        self.lstms: dict[str, list] = {}
        for L in self.enc + self.dec:
            if L.kind == "lstm":
                self.lstms[L.name] = [
                    (w[f"{L.name}.lstm.weight_ih_l{i}"].to(dev, dt).contiguous(),
                     w[f"{L.name}.lstm.weight_hh_l{i}"].to(dev, dt).contiguous(),
                     (w[f"{L.name}.lstm.bias_ih_l{i}"] + w[f"{L.name}.lstm.bias_hh_l{i}"]).to(dev).contiguous())
                    for i in range(cfg.num_lstm_layers)]
        if seanet_only:
            return
        self.books = [w[f"quantizer.layers.{i}.codebook.embed"].to(dev).contiguous()
                      for i in range(cfg.num_quantizers)]
        self.book_sq = [b.pow(2).sum(1) for b in self.books]

    # -- convolutions ------------------------------------------------------
    def _conv(self, x, name, k, stride=1, dil=1, act=None, residual=None):
        c = self.cfg
        T = x.shape[1]
        keff = (k - 1) * dil + 1
        total = keff - stride
        n_frames = math.ceil((T - keff + total) / stride + 1) - 1
        extra = n_frames * stride + keff - total - T
        if c.use_causal_conv:
            pl, pr = total, extra
        else:
            pl, pr = total - total // 2, total // 2 + extra
        reflect = c.pad_mode == "reflect"
        if reflect and T <= max(pl, pr):
            # reflection of a signal shorter than the padding: zeros are appended
            # first and the same number of samples is cut after reflecting
            e = max(pl, pr) - T + 1
            xf = F.elu(x.float()) if act == "elu" else x.float()
            xp = F.pad(F.pad(xf, (0, 0, 0, e)).transpose(1, 2), (pl, pr), mode="reflect")
            x = xp[..., :xp.shape[-1] - e].transpose(1, 2).to(x.dtype).contiguous()
            pl, pr, reflect, act = 0, 0, False, None
        norm = self.norms.get(name)
        y = self.run.conv(x, self.convs[name], act=act, stride=stride, pad=pl, pad_right=pr, dil=dil,
                          reflect=reflect, residual=None if norm is not None else residual)
        if norm is not None:
            y = self._group_norm(y, *norm)
            if residual is not None:
                y = y + residual
        return y

    @staticmethod
    def _group_norm(y, g, b, eps=1e-5):
        yf = y.float()
        mean = yf.mean(dim=(1, 2), keepdim=True)
        var = yf.var(dim=(1, 2), unbiased=False, keepdim=True)
        return ((yf - mean) * torch.rsqrt(var + eps) * g + b).to(y.dtype)

    def _conv_t(self, x, name, k, stride, act):
        c = self.cfg
        total = k - stride
        pr = math.ceil(total * c.trim_right_ratio) if c.use_causal_conv else total // 2
        norm = self.norms.get(name)
        if norm is None:
            return self.run.conv_t(x, self.convs[name], stride=stride, pad=total - pr, pad_right=pr, act=act)
        # the norm's statistics cover the untrimmed output
        y = self._group_norm(self.run.conv_t(x, self.convs[name], stride=stride, pad=0, pad_right=0, act=act), *norm)
        return y[:, total - pr:y.shape[1] - pr].contiguous()

    def _res(self, x, L: _Layer):
        c = self.cfg
        short = (self._conv(x, f"{L.name}.shortcut", 1) if c.use_conv_shortcut else x)
        h = self._conv(x, f"{L.name}.block.1", c.residual_kernel_size, dil=L.res_dil, act="elu")
        return self._conv(h, f"{L.name}.block.3", 1, act="elu", residual=short)

    def _stack(self, x, layers):
        act = None
        for L in layers:
            if L.kind == "elu":
                act = "elu"            # fused into the next conv's operand
                continue
            if L.kind == "conv":
                x = self._conv(x, L.name, L.k, L.stride, act=act)
            elif L.kind == "convt":
                x = self._conv_t(x, L.name, L.k, L.stride, act)
            elif L.kind == "res":
                x = self._res(x, L)
            elif L.kind == "lstm":
                x = (self.run.lstm(x, self.lstms[L.name]) + x).contiguous()
            act = None
        return x

    # -- quantiser ---------------------------------------------------------
    @torch.no_grad()
    def quantize(self, z: torch.Tensor, n_q: int) -> torch.Tensor:
        """z [B, T, D] -> codes [B, n_q, T]."""
        B, T, D = z.shape
        r = z.reshape(B * T, D).float()
        codes = []
        for book, sq in zip(self.books[:n_q], self.book_sq[:n_q]):
            idx = (2 * r @ book.t() - sq).argmax(1)
            r = r - book[idx]
            codes.append(idx.view(B, T))
        return torch.stack(codes, 1)

    @torch.no_grad()
    def dequantize(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, n, T] -> [B, T, D] fp32."""
        codes = codes.to(self.device).long()
        return sum(self.books[i][codes[:, i]] for i in range(codes.shape[1]))

    # -- frames ------------------------------------------------------------
    @torch.no_grad()
    def encode_latents(self, audio: torch.Tensor) -> torch.Tensor:
        """audio [B, C, samples] -> [B, frames, hidden] fp32."""
        x = audio.to(self.device, self.dtype).transpose(1, 2).contiguous()
        return self._stack(x, self.enc).float()

    @torch.no_grad()
    def decode_latents(self, z: torch.Tensor) -> torch.Tensor:
        """[B, frames, hidden] -> audio [B, C, samples] fp32."""
        y = self._stack(z.to(self.device, self.dtype).contiguous(), self.dec)
        return y.float().transpose(1, 2)

    def _encode_frame(self, x: torch.Tensor, n_q: int):
        scale = None
        if self.cfg.normalize:
            mono = x.mean(1, keepdim=True)
            scale = mono.pow(2).mean(-1, keepdim=True).sqrt() + 1e-8
            x = x / scale
            scale = scale.view(-1, 1)
        return self.quantize(self.encode_latents(x), n_q), scale

    @torch.no_grad()
    def encode(self, audio, bandwidth: float | None = None):
        """audio [samples] / [C, samples] / [B, C, samples] at the model rate ->
        (codes [chunks, B, n_q, frames], scales (one [B, 1] or None per chunk),
        last_frame_pad_length), the layout of transformers' EncodecModel.encode.
        ``bandwidth`` (kbps) picks n_q; None: the smallest target bandwidth."""
        c = self.cfg
        x = torch.as_tensor(audio, dtype=torch.float32)
        while x.dim() < 3:
            x = x[None]
        x = x.to(self.device)
        bw = c.target_bandwidths[0] if bandwidth is None else bandwidth
        n_q = c.quantizers_for(bw)
        L = x.shape[-1]
        chunk, stride = (L, L) if c.chunk_length is None else (c.chunk_length, c.chunk_stride)
        frames, scales = [], []
        for off in range(0, L, stride):
            codes, scale = self._encode_frame(x[..., off:off + chunk], n_q)
            frames.append(codes)
            scales.append(scale)
        pad = frames[0].shape[-1] - frames[-1].shape[-1]
        if pad > 0:
            frames[-1] = F.pad(frames[-1], (0, pad))
        return torch.stack(frames), scales, pad

    @torch.no_grad()
    def decode(self, codes: torch.Tensor, scales=None, last_frame_pad_length: int = 0,
               length: int | None = None) -> torch.Tensor:
        """Inverse of ``encode`` -> audio [B, C, samples] fp32 (cut to ``length``)."""
        c = self.cfg
        if codes.dim() == 3:
            codes = codes[None]
        scales = scales if scales is not None else [None] * codes.shape[0]
        outs = []
        for i in range(codes.shape[0]):
            fr = codes[i]
            if i == codes.shape[0] - 1 and last_frame_pad_length > 0:
                fr = fr[..., :-last_frame_pad_length]
            y = self.decode_latents(self.dequantize(fr))
            if scales[i] is not None:
                y = y * scales[i].to(y.device).view(-1, 1, 1)
            outs.append(y)
        if c.chunk_length is None:
            if len(outs) != 1:
                raise ValueError(f"expected one frame, got {len(outs)}")
            y = outs[0]
        else:
            y = _overlap_add(outs, c.chunk_stride or 1)
        return y if length is None else y[..., :length]


def _overlap_add(frames: list, stride: int) -> torch.Tensor:
    """Triangular-window overlap-add of decoded chunks."""
    n = frames[0].shape[-1]
    total = stride * (len(frames) - 1) + frames[-1].shape[-1]
    t = torch.linspace(0, 1, n + 2, device=frames[0].device)[1:-1]
    wgt = 0.5 - (t - 0.5).abs()
    out = torch.zeros(*frames[0].shape[:-1], total, device=frames[0].device)
    den = torch.zeros(total, device=frames[0].device)
    for i, f in enumerate(frames):
        m = f.shape[-1]
        out[..., i * stride:i * stride + m] += wgt[:m] * f
        den[i * stride:i * stride + m] += wgt[:m]
    return out / den


def random_weights(cfg: EncodecConfig, seed: int = 0) -> dict:
    """Seeded transformers-named weights (weight-normalised g / v pairs, or
    plain weights + GroupNorm affine for time_group_norm), with small residual
    branches so activations stay O(1) through the stack."""
    g = torch.Generator().manual_seed(seed)
    w = {}
    wn = cfg.norm_type == "weight_norm"

    def conv(name, o, c, k, transposed=False, gain=1.0):
        shape = (c, o, k) if transposed else (o, c, k)
        t = gain * torch.randn(*shape, generator=g) / math.sqrt(c * k)
        if wn:
            w[name + ".conv.parametrizations.weight.original1"] = t
            w[name + ".conv.parametrizations.weight.original0"] = t.reshape(t.shape[0], -1).norm(dim=1).reshape(
                -1, 1, 1) * (0.8 + 0.4 * torch.rand(t.shape[0], 1, 1, generator=g))
        else:
            w[name + ".conv.weight"] = t
            w[name + ".norm.weight"] = 1 + 0.1 * torch.randn(o, generator=g)
            w[name + ".norm.bias"] = 0.1 * torch.randn(o, generator=g)
        w[name + ".conv.bias"] = 0.05 * torch.randn(o, generator=g)

    def lstm(name, d):
        for i in range(cfg.num_lstm_layers):
            for kind in ("ih", "hh"):
                w[f"{name}.lstm.weight_{kind}_l{i}"] = torch.randn(4 * d, d, generator=g) / math.sqrt(d)
                w[f"{name}.lstm.bias_{kind}_l{i}"] = 0.1 * torch.randn(4 * d, generator=g)

    enc, dec = _layout(cfg)
    d = cfg.num_filters
    for L in enc:
        if L.kind == "conv" and L.name == "encoder.layers.0":
            conv(L.name, d, cfg.audio_channels, L.k)
        elif L.kind == "res":
            h = d // cfg.compress
            conv(L.name + ".block.1", h, d, cfg.residual_kernel_size)
            conv(L.name + ".block.3", d, h, 1, gain=0.3)
            if cfg.use_conv_shortcut:
                conv(L.name + ".shortcut", d, d, 1)
        elif L.kind == "conv" and L.stride > 1:
            conv(L.name, 2 * d, d, L.k)
            d *= 2
        elif L.kind == "lstm":
            lstm(L.name, d)
        elif L.kind == "conv":
            conv(L.name, cfg.hidden_size, d, L.k)
    d = cfg.num_filters * 2 ** len(cfg.upsampling_ratios)
    for L in dec:
        if L.kind == "conv" and L.name == "decoder.layers.0":
            conv(L.name, d, cfg.hidden_size, L.k)
        elif L.kind == "lstm":
            lstm(L.name, d)
        elif L.kind == "convt":
            conv(L.name, d // 2, d, L.k, transposed=True)
            d //= 2
        elif L.kind == "res":
            h = d // cfg.compress
            conv(L.name + ".block.1", h, d, cfg.residual_kernel_size)
            conv(L.name + ".block.3", d, h, 1, gain=0.3)
            if cfg.use_conv_shortcut:
                conv(L.name + ".shortcut", d, d, 1)
        elif L.kind == "conv":
            conv(L.name, cfg.audio_channels, d, L.k)
    for i in range(cfg.num_quantizers):
        p = f"quantizer.layers.{i}.codebook."
        e = torch.randn(cfg.codebook_size, cfg.codebook_dim, generator=g)
        w[p + "embed"] = e
        w[p + "embed_avg"] = e.clone()
        w[p + "cluster_size"] = torch.ones(cfg.codebook_size)
        w[p + "inited"] = torch.ones(1)
    return w
