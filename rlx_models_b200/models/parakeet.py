"""Parakeet FastConformer speech recognition (CTC head).

    features  log-mel (80 bins, 25 ms Hann window in a 512-point FFT, 10 ms hop,
              pre-emphasis 0.97, power spectrum, Slaney mel, log(x + 2^-24),
              per-bin mean / std over the valid frames)
    subsample conv2d stride 2 (ReLU), then (depthwise 3x3 stride 2 + pointwise 1x1 + ReLU)
              per further factor of 2 -> [B, T / 8, C * mel / 8] -> linear -> H,
              scaled by sqrt(H)
    block     x += 0.5 FF1(LN x)                       (Macaron half-step FFN, SiLU)
              x += MHSA(LN x) with relative positions  (Transformer-XL: scores
                   (q + u) k^T + rel_shift((q + v) (W_pos p)^T), p = sinusoids of
                   the distances T-1 .. -(T-1))
              x += Conv(LN x)                          (pointwise -> GLU -> depthwise k
                   -> BatchNorm -> SiLU -> pointwise)
              x += 0.5 FF2(LN x); x = LN x
    head      1x1 conv -> vocab (+ blank); greedy CTC: argmax per frame, merge
              repeats, drop blanks

Linear layers run on the package's GEMM (bf16 on CUDA), the rest in torch.
transformers' ParakeetForCTC is the CPU oracle (its feature extractor needs
librosa, absent here; the features follow its definition).

Reference: crates/rlx-parakeet (the FastConformer encoder; its TDT transducer
decoder is not built here).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .flux_text import _linear

LOG_GUARD = 2.0 ** -24
NORM_EPS = 1e-5


@dataclass
class ParakeetConfig:
    hidden_size: int = 1024
    num_hidden_layers: int = 24
    num_attention_heads: int = 8
    intermediate_size: int = 4096
    hidden_act: str = "silu"
    attention_bias: bool = True
    convolution_bias: bool = True
    conv_kernel_size: int = 9
    subsampling_factor: int = 8
    subsampling_conv_channels: int = 256
    num_mel_bins: int = 80
    subsampling_conv_kernel_size: int = 3
    subsampling_conv_stride: int = 2
    scale_input: bool = True
    vocab_size: int = 1025
    blank_id: int = 1024

    @classmethod
    def from_dict(cls, d: dict) -> "ParakeetConfig":
        enc = dict(d.get("encoder_config") or d)
        kw = {k: enc[k] for k in cls.__dataclass_fields__ if k in enc}
        kw["vocab_size"] = int(d.get("vocab_size", 1025))
        kw["blank_id"] = int(d.get("pad_token_id", kw["vocab_size"] - 1))
        return cls(**kw)


def log_mel_features(audio: torch.Tensor, sr: int = 16000, n_mels: int = 80) -> torch.Tensor:
    """[N] float waveform -> [frames, n_mels] normalised log-mel features."""
    from ..utils.preprocess import mel_filter_bank
    x = audio.float()
    x = torch.cat([x[:1], x[1:] - 0.97 * x[:-1]])
    n_fft, hop, win = 512, 160, 400
    st = torch.stft(x, n_fft, hop_length=hop, win_length=win, window=torch.hann_window(win, periodic=False),
                    return_complex=True, pad_mode="constant")
    power = torch.view_as_real(st).pow(2).sum(-1)  # [n_fft/2 + 1, frames]
    fb = mel_filter_bank(n_fft // 2 + 1, n_mels, 0.0, sr / 2, sr, norm="slaney", mel_scale="slaney")
    mel = torch.log(fb.t() @ power + LOG_GUARD).t()  # [frames, n_mels]
    n = (x.shape[0] + n_fft // 2 * 2 - n_fft) // hop  # valid frames
    mel = mel[: max(n, 1)]
    mean = mel.mean(0, keepdim=True)
    std = ((mel - mean).pow(2).sum(0, keepdim=True) / max(mel.shape[0] - 1, 1)).sqrt()
    return (mel - mean) / (std + NORM_EPS)


class ParakeetCTC:
    def __init__(self, cfg: ParakeetConfig, weights, device="cpu", dtype: torch.dtype | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        get = (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])
        has = lambda n: n in weights  # noqa: E731
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        f32 = lambda t: t.to(self.device, torch.float32).contiguous()  # noqa: E731
        opt = lambda n: dv(get(n)) if has(n) else None  # noqa: E731
        e = "encoder."
        # subsampling convolutions (torch convs, fp32) and the projection
        self.sub = []
        n_sub = int(math.log2(cfg.subsampling_factor))
        for i in range(2 + 3 * (n_sub - 1)):  # conv, relu, then (depthwise, pointwise, relu) per factor 2
            if has(e + f"subsampling.layers.{i}.weight"):
                self.sub.append((i, f32(get(e + f"subsampling.layers.{i}.weight")),
                                 f32(get(e + f"subsampling.layers.{i}.bias"))))
        self.sub_lin = (dv(get(e + "subsampling.linear.weight")), dv(get(e + "subsampling.linear.bias")))
        H = cfg.hidden_size
        self.layers = []
        for li in range(cfg.num_hidden_layers):
            p = e + f"layers.{li}."
            ln = lambda n: (f32(get(p + n + ".weight")), f32(get(p + n + ".bias")))  # noqa: E731
            lin = lambda n: (dv(get(p + n + ".weight")), opt(p + n + ".bias"))  # noqa: E731
            a = p + "self_attn."
            c = p + "conv."
            self.layers.append(dict(
                ln_ff1=ln("norm_feed_forward1"), ln_att=ln("norm_self_att"), ln_conv=ln("norm_conv"),
                ln_ff2=ln("norm_feed_forward2"), ln_out=ln("norm_out"),
                ff1=(lin("feed_forward1.linear1"), lin("feed_forward1.linear2")),
                ff2=(lin("feed_forward2.linear1"), lin("feed_forward2.linear2")),
                qkv=(dv(torch.cat([get(a + f"{n}_proj.weight") for n in "qkv"])),
                     dv(torch.cat([get(a + f"{n}_proj.bias") for n in "qkv"])) if cfg.attention_bias else None),
                o=lin("self_attn.o_proj"), pos=dv(get(a + "relative_k_proj.weight")),
                bias_u=f32(get(a + "bias_u")), bias_v=f32(get(a + "bias_v")),
                pw1=(dv(get(c + "pointwise_conv1.weight").reshape(2 * H, H)), opt(c + "pointwise_conv1.bias")),
                dw=(f32(get(c + "depthwise_conv.weight")), f32(get(c + "depthwise_conv.bias"))
                    if has(c + "depthwise_conv.bias") else None),
                bn=tuple(f32(get(c + f"norm.{n}")) for n in ("weight", "bias", "running_mean", "running_var")),
                pw2=(dv(get(c + "pointwise_conv2.weight").reshape(H, H)), opt(c + "pointwise_conv2.bias"))))
        hw = get("ctc_head.weight")
        self.head = (dv(hw.reshape(hw.shape[0], -1)), dv(get("ctc_head.bias")))

    # -- pieces -----------------------------------------------------------------
    def _subsample(self, feats: torch.Tensor, lengths: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        c = self.cfg
        x = feats.unsqueeze(1).float()  # [B, 1, T, mel]
        k, s = c.subsampling_conv_kernel_size, c.subsampling_conv_stride
        pad = (k - 1) // 2
        cur = lengths.clone()
        for idx, w, b in self.sub:
            if w.shape[-1] == 1:  # pointwise
                x = F.conv2d(x, w, b)
            else:
                groups = 1 if w.shape[1] == x.shape[1] else x.shape[1]
                x = F.conv2d(x, w, b, stride=s, padding=pad, groups=groups)
                cur = (cur + 2 * pad - k) // s + 1
            if w.shape[-1] == 1 or idx == 0:
                x = F.relu(x)
            x = x * (torch.arange(x.shape[2], device=x.device)[None, :] < cur[:, None])[:, None, :, None]
        B, C, T, Fq = x.shape
        x = x.transpose(1, 2).reshape(B, T, C * Fq).to(self.dtype)
        return _linear(x, *self.sub_lin), cur

    def _ln(self, x, p):
        return F.layer_norm(x.float(), (x.shape[-1],), p[0], p[1], 1e-5)

    def _attention(self, ly, x, pos_emb, mask):
        c = self.cfg
        B, T, H = x.shape
        nh = c.num_attention_heads
        D = H // nh
        q, k, v = _linear(x.to(self.dtype), *ly["qkv"]).float().split(H, -1)
        q, k, v = (t.view(B, T, nh, D) for t in (q, k, v))
        p = _linear(pos_emb.to(self.dtype), ly["pos"]).float().view(-1, nh, D)  # [2T - 1, nh, D]
        ac = torch.einsum("bthd,bshd->bhts", q + ly["bias_u"], k)
        bd = torch.einsum("bthd,shd->bhts", q + ly["bias_v"], p)  # distance index s: T-1 .. -(T-1)
        # relative shift: row t takes distances t - s for s = 0 .. T-1, i.e. columns T-1-t+s
        idx = (T - 1 - torch.arange(T, device=x.device))[:, None] + torch.arange(T, device=x.device)[None, :]
        bd = bd.gather(-1, idx[None, None].expand(B, nh, T, T))
        s = (ac + bd) / math.sqrt(D)
        if mask is not None:
            s = s.masked_fill(~mask[:, None], float("-inf"))
        pr = torch.softmax(s, -1)
        if mask is not None:
            pr = torch.nan_to_num(pr)
        o = torch.einsum("bhts,bshd->bthd", pr, v).reshape(B, T, H)
        return _linear(o.to(self.dtype), *ly["o"]).float()

    def _conv(self, ly, x, valid):
        B, T, H = x.shape
        y = _linear(x.to(self.dtype), *ly["pw1"]).float()
        y = F.glu(y, dim=-1)
        y = y * valid[..., None]
        y = F.conv1d(y.transpose(1, 2), ly["dw"][0], ly["dw"][1], padding=(ly["dw"][0].shape[-1] - 1) // 2,
                     groups=H)
        w, b, rm, rv = ly["bn"]
        y = (y - rm[None, :, None]) * torch.rsqrt(rv[None, :, None] + 1e-5) * w[None, :, None] + b[None, :, None]
        y = F.silu(y).transpose(1, 2)
        return _linear(y.to(self.dtype), *ly["pw2"]).float()

    def _ff(self, pr, x):
        h = F.silu(_linear(x.to(self.dtype), *pr[0]).float())
        return _linear(h.to(self.dtype), *pr[1]).float()

    def _positions(self, T: int) -> torch.Tensor:
        H = self.cfg.hidden_size
        inv = 1.0 / (10000.0 ** (torch.arange(0, H, 2, device=self.device).float() / H))
        dist = torch.arange(T - 1, -T, -1, device=self.device).float()
        ang = dist[:, None] * inv[None, :]
        return torch.stack([ang.sin(), ang.cos()], -1).reshape(2 * T - 1, H)

    # -- forward ------------------------------------------------------------------
    @torch.no_grad()
    def logits(self, feats: torch.Tensor, lengths: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """feats [B, T, mel] normalised log-mel -> (CTC logits [B, T', V] fp32, output lengths [B])."""
        c = self.cfg
        feats = feats.to(self.device)
        B = feats.shape[0]
        lengths = (torch.full((B,), feats.shape[1], dtype=torch.long) if lengths is None
                   else torch.as_tensor(lengths)).to(self.device)
        x, out_len = self._subsample(feats, lengths)
        x = x.float() * (math.sqrt(c.hidden_size) if c.scale_input else 1.0)
        T = x.shape[1]
        valid = (torch.arange(T, device=self.device)[None, :] < out_len[:, None]).float()
        mask = (valid[:, :, None] * valid[:, None, :]).bool() if bool((out_len < T).any()) else None
        pos = self._positions(T)
        for ly in self.layers:
            x = x + 0.5 * self._ff(ly["ff1"], self._ln(x, ly["ln_ff1"]))
            x = x + self._attention(ly, self._ln(x, ly["ln_att"]), pos, mask)
            x = x + self._conv(ly, self._ln(x, ly["ln_conv"]), valid if mask is not None else torch.ones_like(valid))
            x = x + 0.5 * self._ff(ly["ff2"], self._ln(x, ly["ln_ff2"]))
            x = self._ln(x, ly["ln_out"])
        return _linear(x.to(self.dtype), *self.head).float(), out_len

    def greedy(self, feats: torch.Tensor, lengths=None) -> list[list[int]]:
        """Greedy CTC decoding: per-frame argmax, repeats merged, blanks dropped."""
        lg, n = self.logits(feats, lengths)
        out = []
        for b in range(lg.shape[0]):
            best = lg[b, : int(n[b])].argmax(-1).tolist()
            seq, prev = [], None
            for t in best:
                if t != prev and t != self.cfg.blank_id:
                    seq.append(t)
                prev = t
            out.append(seq)
        return out


class ParakeetTranscriber:
    """``transcribe(audio, sample_rate)`` over a ParakeetCTC model."""

    def __init__(self, model: ParakeetCTC, tokenizer=None):
        self.model, self.tokenizer = model, tokenizer

    def transcribe(self, audio, sample_rate: int = 16000):
        a = torch.as_tensor(audio, dtype=torch.float32)
        if a.dim() > 1:
            a = a.mean(-1)
        if sample_rate != 16000:
            a = F.interpolate(a[None, None], scale_factor=16000 / sample_rate, mode="linear",
                              align_corners=False)[0, 0]
        ids = self.model.greedy(log_mel_features(a, 16000, self.model.cfg.num_mel_bins)[None])[0]
        return self.tokenizer.decode(ids) if self.tokenizer is not None else ids
