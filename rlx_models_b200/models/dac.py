"""DAC (Descript Audio Codec): a convolutional audio autoencoder with a
residual vector quantiser, 16 / 24 / 44.1 kHz mono.

    encoder  conv(1 -> d, k7) -> [res(d1), res(d3), res(d9), snake, conv(k 2s, stride s)] per
             downsampling ratio s (channels double each block) -> snake -> conv(k3) -> z [T, H]
    res(dl)  x + conv1x1(snake(conv(k7, dilation dl)(snake(x))))
    RVQ      per codebook i: p = in_proj_i(r) (H -> D); code = argmax cos(p, codebook_i);
             q_i = out_proj_i(codebook_i[code]) (D -> H); r -= q_i; z_q = sum_i q_i
    decoder  conv(H -> d, k7) -> [snake, convT(k 2s, stride s), res(1), res(3), res(9)] per
             upsampling ratio (channels halve) -> snake -> conv(k7, -> 1) -> tanh
    snake(x) = x + sin(alpha x)^2 / (alpha + 1e-9), alpha per channel

Every convolution runs channels-last ([B, T, C]) as a GEMM on the tcgen05
linear: ``ops.act_im2col`` builds the operand with the preceding Snake fused
in, a 1x1 conv is a plain linear (the residual add rides in its epilogue), and
the transposed convolutions are one GEMM into fp32 taps followed by
``ops.convt_fold`` (overlap-add, bias and crop in one pass). Weight
normalisation (``weight_g`` / ``weight_v`` or ``parametrizations.weight.original0/1``)
is folded into plain weights at load. The quantiser is a few [T, 1024] x [1024, 8]
products and stays in fp32 torch. On CPU the same layout code runs in fp32
against the torch statements of the two kernels (``ops/reference.py``).

Checkpoint names: transformers' DacModel layout and the original Descript
layout (``encoder.block.N.block.M...``, ``decoder.model.N...``).

Reference: crates/rlx-dac/src/codec.rs:130-185 (pad to the hop, encode, decode,
roundtrip), crates/rlx-dac/src/build.rs:110-211 (weight names),
crates/rlx-dac/src/quantize.rs (RVQ with l2-normalised codes),
crates/rlx-dac/src/config.rs:41-90 (the three released configs).
"""
from __future__ import annotations

import math
import re
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .codec_common import ConvRunner, GemmConv, fold_weight_norm


@dataclass
class DacConfig:
    encoder_hidden_size: int = 64
    downsampling_ratios: list = field(default_factory=lambda: [2, 4, 8, 8])
    decoder_hidden_size: int = 1536
    upsampling_ratios: list = field(default_factory=lambda: [8, 8, 4, 2])
    n_codebooks: int = 9
    codebook_size: int = 1024
    codebook_dim: int = 8
    hidden_size: int = 1024
    sampling_rate: int = 44100
    hop_length: int = 512

    @classmethod
    def from_dict(cls, d: dict) -> "DacConfig":
        """transformers' DacConfig keys, or the Descript / reference names
        (encoder_dim, encoder_rates, decoder_dim, decoder_rates, latent_dim, sample_rate)."""
        g = lambda a, b, dflt: d.get(a, d.get(b, dflt))  # noqa: E731
        down = list(g("downsampling_ratios", "encoder_rates", [2, 4, 8, 8]))
        return cls(encoder_hidden_size=int(g("encoder_hidden_size", "encoder_dim", 64)),
                   downsampling_ratios=down,
                   decoder_hidden_size=int(g("decoder_hidden_size", "decoder_dim", 1536)),
                   upsampling_ratios=list(g("upsampling_ratios", "decoder_rates", [8, 8, 4, 2])),
                   n_codebooks=int(d.get("n_codebooks", 9)), codebook_size=int(d.get("codebook_size", 1024)),
                   codebook_dim=int(d.get("codebook_dim", 8)),
                   hidden_size=int(g("hidden_size", "latent_dim", 1024)),
                   sampling_rate=int(g("sampling_rate", "sample_rate", 44100)),
                   hop_length=int(d.get("hop_length", math.prod(down))))


_RES = ("snake1", "conv1", "snake2", "conv2")


def _descript_name(name: str, n_enc: int, n_dec: int) -> str:
    """Original Descript checkpoint name -> transformers' DacModel name."""
    m = re.match(r"encoder\.block\.(\d+)\.(.*)$", name)
    if m:
        i, rest = int(m.group(1)), m.group(2)
        if i == 0:
            return "encoder.conv1." + rest
        if i == n_enc + 1:
            return "encoder.snake1." + rest
        if i == n_enc + 2:
            return "encoder.conv2." + rest
        r = re.match(r"block\.(\d+)\.(.*)$", rest)
        j, tail = int(r.group(1)), r.group(2)
        if j < 3:
            u = re.match(r"block\.(\d+)\.(.*)$", tail)
            return f"encoder.block.{i - 1}.res_unit{j + 1}.{_RES[int(u.group(1))]}.{u.group(2)}"
        return f"encoder.block.{i - 1}.{'snake1' if j == 3 else 'conv1'}.{tail}"
    m = re.match(r"decoder\.model\.(\d+)\.(.*)$", name)
    if m:
        i, rest = int(m.group(1)), m.group(2)
        if i == 0:
            return "decoder.conv1." + rest
        if i == n_dec + 1:
            return "decoder.snake1." + rest
        if i == n_dec + 2:
            return "decoder.conv2." + rest
        r = re.match(r"block\.(\d+)\.(.*)$", rest)
        j, tail = int(r.group(1)), r.group(2)
        if j >= 2:
            u = re.match(r"block\.(\d+)\.(.*)$", tail)
            return f"decoder.block.{i - 1}.res_unit{j - 1}.{_RES[int(u.group(1))]}.{u.group(2)}"
        return f"decoder.block.{i - 1}.{'snake1' if j == 0 else 'conv_t1'}.{tail}"
    return name


def fold_weights(weights, cfg: DacConfig) -> dict:
    """Plain fp32 tensors under transformers' names, weight norm folded."""
    get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
    keys = list(weights.keys())
    descript = any(k.startswith("decoder.model.") for k in keys)
    ne, nd = len(cfg.downsampling_ratios), len(cfg.upsampling_ratios)
    return fold_weight_norm({(_descript_name(k, ne, nd) if descript else k): get(k) for k in keys})


class DacModel:
    def __init__(self, cfg: DacConfig, weights, device="cpu"):
        self.cfg = cfg
        self.run = ConvRunner(device)
        self.device, self.dtype = self.run.device, self.run.dtype
        w = fold_weights(weights, cfg)
        dt, dev = self.dtype, self.device
        self.convs: dict[str, GemmConv] = {}
        self.alpha: dict[str, torch.Tensor] = {}
        for n, t in w.items():
            if n.endswith(".alpha"):
                self.alpha[n[:-len(".alpha")]] = t.reshape(-1).to(dev, torch.float32).contiguous()
            elif n.endswith(".weight") and (n.startswith("encoder.") or n.startswith("decoder.")):
                base = n[:-len(".weight")]
                self.convs[base] = GemmConv(t, w.get(base + ".bias"), base.endswith("conv_t1"), dt, dev)
        f32 = lambda t: t.to(dev, torch.float32).contiguous()  # noqa: E731
        self.quant = []
        for i in range(cfg.n_codebooks):
            p = f"quantizer.quantizers.{i}."
            self.quant.append(dict(
                w_in=f32(w[p + "in_proj.weight"].reshape(cfg.codebook_dim, -1)), b_in=f32(w[p + "in_proj.bias"]),
                w_out=f32(w[p + "out_proj.weight"].reshape(cfg.hidden_size, -1)), b_out=f32(w[p + "out_proj.bias"]),
                book=f32(w[p + "codebook.weight"])))
            self.quant[-1]["book_n"] = F.normalize(self.quant[-1]["book"], dim=1)

    # -- primitives --------------------------------------------------------
    def _conv(self, x: torch.Tensor, name: str, snake: str | None = None, stride: int = 1, pad: int = 0,
              dil: int = 1, residual: torch.Tensor | None = None) -> torch.Tensor:
        """x [B, T, C] -> [B, T_out, O] of conv ``name`` after the Snake ``snake``."""
        return self.run.conv(x, self.convs[name], act="snake" if snake is not None else None,
                             alpha=self.alpha[snake] if snake is not None else None, stride=stride, pad=pad,
                             dil=dil, residual=residual)

    def _conv_t(self, x: torch.Tensor, name: str, snake: str, stride: int) -> torch.Tensor:
        return self.run.conv_t(x, self.convs[name], stride=stride, pad=math.ceil(stride / 2), act="snake",
                               alpha=self.alpha[snake])

    def _res(self, x: torch.Tensor, p: str, dil: int) -> torch.Tensor:
        h = self._conv(x, p + "conv1", p + "snake1", pad=3 * dil, dil=dil)
        return self._conv(h, p + "conv2", p + "snake2", residual=x)

    # -- encoder / decoder -------------------------------------------------
    @torch.no_grad()
    def encode_latents(self, audio: torch.Tensor) -> torch.Tensor:
        """audio [B, samples] (a multiple of the hop) -> z [B, frames, hidden] fp32."""
        x = audio.to(self.device, self.dtype)[:, :, None].contiguous()
        x = self._conv(x, "encoder.conv1", pad=3)
        for i, s in enumerate(self.cfg.downsampling_ratios):
            p = f"encoder.block.{i}."
            for u, dil in ((1, 1), (2, 3), (3, 9)):
                x = self._res(x, f"{p}res_unit{u}.", dil)
            x = self._conv(x, p + "conv1", p + "snake1", stride=s, pad=math.ceil(s / 2))
        return self._conv(x, "encoder.conv2", "encoder.snake1", pad=1).float()

    @torch.no_grad()
    def quantize(self, z: torch.Tensor, n_quantizers: int | None = None):
        """z [B, T, H] -> (codes [B, n, T] int64, z_q [B, T, H] fp32)."""
        nq = self.cfg.n_codebooks if n_quantizers is None else min(n_quantizers, self.cfg.n_codebooks)
        B, T, H = z.shape
        r = z.reshape(B * T, H).float()
        zq = torch.zeros_like(r)
        codes = []
        for q in self.quant[:nq]:
            p = r @ q["w_in"].t() + q["b_in"]
            idx = (F.normalize(p, dim=1) @ q["book_n"].t()).argmax(1)
            qi = q["book"][idx] @ q["w_out"].t() + q["b_out"]
            zq = zq + qi
            r = r - qi
            codes.append(idx.view(B, T))
        return torch.stack(codes, 1), zq.view(B, T, H)

    @torch.no_grad()
    def dequantize(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, n, T] -> z_q [B, T, H] fp32 (sum of the first n codebooks)."""
        codes = codes.to(self.device).long()
        B, n, T = codes.shape
        zq = torch.zeros(B * T, self.cfg.hidden_size, device=self.device)
        for i in range(n):
            q = self.quant[i]
            zq = zq + q["book"][codes[:, i].reshape(-1)] @ q["w_out"].t() + q["b_out"]
        return zq.view(B, T, -1)

    def _dec_body(self, zq: torch.Tensor) -> torch.Tensor:
        x = self._conv(zq.to(self.device, self.dtype).contiguous(), "decoder.conv1", pad=3)
        for i, s in enumerate(self.cfg.upsampling_ratios):
            p = f"decoder.block.{i}."
            x = self._conv_t(x, p + "conv_t1", p + "snake1", s)
            for u, dil in ((1, 1), (2, 3), (3, 9)):
                x = self._res(x, f"{p}res_unit{u}.", dil)
        return x

    @torch.no_grad()
    def decode_latents(self, zq: torch.Tensor) -> torch.Tensor:
        """z_q [B, T, H] -> audio [B, samples] fp32."""
        y = self._conv(self._dec_body(zq), "decoder.conv2", "decoder.snake1", pad=3)
        return torch.tanh(y.float())[..., 0]

    # -- codec API ---------------------------------------------------------
    def _pad(self, audio: torch.Tensor) -> torch.Tensor:
        audio = torch.as_tensor(audio, dtype=torch.float32)
        if audio.dim() == 1:
            audio = audio[None]
        return F.pad(audio, (0, (-audio.shape[-1]) % self.cfg.hop_length))

    @torch.no_grad()
    def encode(self, audio, n_quantizers: int | None = None) -> torch.Tensor:
        """Mono PCM [samples] or [B, samples] at the model rate -> codes [B, n, frames]
        (right-padded to a multiple of the hop)."""
        return self.quantize(self.encode_latents(self._pad(audio)), n_quantizers)[0]

    @torch.no_grad()
    def decode(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, n, frames] -> PCM [B, samples] fp32."""
        return self.decode_latents(self.dequantize(codes))

    @torch.no_grad()
    def roundtrip(self, audio, n_quantizers: int | None = None):
        """(codes, reconstruction trimmed to the input length)."""
        a = torch.as_tensor(audio, dtype=torch.float32)
        n = a.shape[-1]
        codes = self.encode(a, n_quantizers)
        return codes, self.decode(codes)[..., :n]


def random_weights(cfg: DacConfig, seed: int = 0, weight_norm: bool = False) -> dict:
    """Seeded weights under transformers' names (weight-normalised g / v pairs
    when ``weight_norm``), scaled so activations stay O(1) through the stack."""
    g = torch.Generator().manual_seed(seed)
    w = {}

    def conv(name, o, c, k, transposed=False, gain=1.0):
        shape = (c, o, k) if transposed else (o, c, k)
        t = gain * torch.randn(*shape, generator=g) / math.sqrt(c * k)
        if weight_norm:
            w[name + ".weight_v"] = t
            w[name + ".weight_g"] = t.reshape(t.shape[0], -1).norm(dim=1).reshape(-1, 1, 1) * (
                0.8 + 0.4 * torch.rand(t.shape[0], 1, 1, generator=g))
        else:
            w[name + ".weight"] = t
        w[name + ".bias"] = 0.05 * torch.randn(o, generator=g)

    def snake(name, c):
        w[name + ".alpha"] = (0.5 + torch.rand(1, c, 1, generator=g))

    def res(p, c):
        snake(p + "snake1", c)
        conv(p + "conv1", c, c, 7)
        snake(p + "snake2", c)
        conv(p + "conv2", c, c, 1, gain=0.3)       # small residual branches, as in trained codecs

    d = cfg.encoder_hidden_size
    conv("encoder.conv1", d, 1, 7)
    for i, s in enumerate(cfg.downsampling_ratios):
        p = f"encoder.block.{i}."
        for u in (1, 2, 3):
            res(f"{p}res_unit{u}.", d)
        snake(p + "snake1", d)
        conv(p + "conv1", 2 * d, d, 2 * s)
        d *= 2
    snake("encoder.snake1", d)
    conv("encoder.conv2", cfg.hidden_size, d, 3)
    d = cfg.decoder_hidden_size
    conv("decoder.conv1", d, cfg.hidden_size, 7)
    for i, s in enumerate(cfg.upsampling_ratios):
        p = f"decoder.block.{i}."
        snake(p + "snake1", d)
        conv(p + "conv_t1", d // 2, d, 2 * s, transposed=True)
        d //= 2
        for u in (1, 2, 3):
            res(f"{p}res_unit{u}.", d)
    snake("decoder.snake1", d)
    conv("decoder.conv2", 1, d, 7)
    for i in range(cfg.n_codebooks):
        p = f"quantizer.quantizers.{i}."
        conv(p + "in_proj", cfg.codebook_dim, cfg.hidden_size, 1)
        conv(p + "out_proj", cfg.hidden_size, cfg.codebook_dim, 1)
        w[p + "codebook.weight"] = torch.randn(cfg.codebook_size, cfg.codebook_dim, generator=g)
    return w
