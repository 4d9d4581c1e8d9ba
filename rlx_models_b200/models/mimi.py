"""Mimi (Kyutai's streaming speech codec, 24 kHz -> 12.5 Hz): the SEANet
convolution stacks of EnCodec without their LSTMs, a causal Transformer on each
side, a stride-2 resampling conv pair, and a split residual vector quantiser.

    encode   SEANet encoder (25 Hz, hidden 512) -> Transformer (LayerNorm, RoPE,
             causal attention over a sliding window of 250 frames, LayerScale on both
             residual branches, GELU MLP) -> downsample conv (k 4, stride 2, replicate
             padding on the left) -> split RVQ: one semantic stage + up to 31 acoustic
             stages, each group with a 1x1 input projection (512 -> 256) and Euclidean
             codebooks (embed = embed_sum / max(cluster_usage, 1e-5))
    decode   codebook sums -> per-group 1x1 output projection (256 -> 512) -> depthwise
             transposed conv (k 4, stride 2) -> Transformer -> SEANet decoder

The SEANet convolutions run on the shared codec blocks (``models/encodec.py`` /
``codec_common.py``: ELU fused into each conv's operand, GEMMs on the tcgen05
linear); the Transformer's linears run on the tcgen05 GEMM in bf16 with SDPA
attention; the resampling convs and the quantiser's distance products stay in
torch.

Checkpoint names: transformers' MimiModel.

Reference: crates/rlx-mimi (the Mimi codec used by the reference's Kyutai TTS
and Moshi-style runners); transformers' MimiModel is the CPU oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .encodec import EncodecConfig, EncodecModel
from .flux_text import _linear


@dataclass
class MimiConfig:
    sampling_rate: int = 24000
    audio_channels: int = 1
    hidden_size: int = 512
    num_filters: int = 64
    num_residual_layers: int = 1
    upsampling_ratios: list = field(default_factory=lambda: [8, 6, 5, 4])
    kernel_size: int = 7
    last_kernel_size: int = 3
    residual_kernel_size: int = 3
    dilation_growth_rate: int = 2
    use_causal_conv: bool = True
    pad_mode: str = "constant"
    compress: int = 2
    trim_right_ratio: float = 1.0
    use_conv_shortcut: bool = False
    codebook_size: int = 2048
    codebook_dim: int = 256
    num_quantizers: int = 32
    num_semantic_quantizers: int = 1
    vector_quantization_hidden_dimension: int = 256
    upsample_groups: int = 512
    num_hidden_layers: int = 8
    intermediate_size: int = 2048
    num_attention_heads: int = 8
    num_key_value_heads: int = 8
    head_dim: int = 64
    hidden_act: str = "gelu"
    norm_eps: float = 1e-5
    sliding_window: int = 250
    rope_theta: float = 10000.0
    frame_rate: float = 12.5

    @classmethod
    def from_dict(cls, d: dict) -> "MimiConfig":
        names = set(cls.__dataclass_fields__)
        kw = {k: v for k, v in d.items() if k in names and v is not None}
        rp = d.get("rope_parameters") or {}
        if isinstance(rp, dict) and rp.get("rope_theta"):
            kw["rope_theta"] = float(rp["rope_theta"])
        if d.get("_frame_rate"):
            kw["frame_rate"] = float(d["_frame_rate"])
        return cls(**kw)

    @property
    def encodec_frame_rate(self) -> int:
        return math.ceil(self.sampling_rate / math.prod(self.upsampling_ratios))

    def seanet(self) -> EncodecConfig:
        return EncodecConfig.from_dict({**self.__dict__, "upsampling_ratios": list(self.upsampling_ratios)})


def _rope(x, inv, pos):
    """Half-split rotary embedding of x [B, nh, T, hd] at positions pos [T]."""
    ang = pos[:, None].float() * inv[None]
    cos, sin = torch.cat([ang.cos()] * 2, -1), torch.cat([ang.sin()] * 2, -1)
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], -1)
    return x * cos + rot * sin


class MimiModel:
    def __init__(self, cfg: MimiConfig, weights, device="cpu"):
        self.cfg = cfg
        self.seanet = EncodecModel(cfg.seanet(), weights, device=device, seanet_only=True)
        self.device, self.dtype = self.seanet.device, self.seanet.dtype
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        dev, dt = self.device, self.dtype
        f32 = lambda n: get(n).to(dev, torch.float32).contiguous()  # noqa: E731
        lw = lambda n: get(n).to(dev, dt).contiguous()  # noqa: E731
        self.tf = {}
        for side in ("encoder_transformer", "decoder_transformer"):
            layers = []
            for i in range(cfg.num_hidden_layers):
                p = f"{side}.layers.{i}."
                layers.append(dict(
                    qkv=torch.cat([get(p + f"self_attn.{n}_proj.weight") for n in "qkv"]).to(dev, dt).contiguous(),
                    o=lw(p + "self_attn.o_proj.weight"),
                    ln1=(f32(p + "input_layernorm.weight"), f32(p + "input_layernorm.bias")),
                    ln2=(f32(p + "post_attention_layernorm.weight"), f32(p + "post_attention_layernorm.bias")),
                    fc1=lw(p + "mlp.fc1.weight"), fc2=lw(p + "mlp.fc2.weight"),
                    s1=f32(p + "self_attn_layer_scale.scale"), s2=f32(p + "mlp_layer_scale.scale")))
            self.tf[side] = layers
        self.inv = 1.0 / cfg.rope_theta ** (torch.arange(0, cfg.head_dim, 2, device=dev).float() / cfg.head_dim)
        self.down_w = f32("downsample.conv.weight")
        self.up_w = f32("upsample.conv.weight")
        self.groups = []
        for name, n in (("semantic", cfg.num_semantic_quantizers),
                        ("acoustic", cfg.num_quantizers - cfg.num_semantic_quantizers)):
            p = f"quantizer.{name}_residual_vector_quantizer."
            books = []
            for i in range(n):
                q = f"{p}layers.{i}.codebook."
                books.append(f32(q + "embed_sum") / f32(q + "cluster_usage").clamp(min=1e-5)[:, None])
            self.groups.append(dict(inp=f32(p + "input_proj.weight")[..., 0], out=f32(p + "output_proj.weight")[..., 0],
                                    books=books, sq=[b.pow(2).sum(1) for b in books]))

    # -- transformer -------------------------------------------------------
    def _transformer(self, x: torch.Tensor, side: str) -> torch.Tensor:
        """x [B, T, H] fp32 -> [B, T, H] fp32 (causal, sliding window)."""
        c = self.cfg
        B, T, H = x.shape
        nh, nkv, hd = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        pos = torch.arange(T, device=self.device)
        rel = pos[:, None] - pos[None, :]
        mask = (rel >= 0) & (rel < c.sliding_window)
        lin = lambda t, w: _linear(t.reshape(-1, t.shape[-1]).to(self.dtype).contiguous(), w).float()  # noqa: E731
        for L in self.tf[side]:
            h = F.layer_norm(x, (H,), *L["ln1"], c.norm_eps)
            qkv = lin(h, L["qkv"]).view(B, T, -1)
            q, k, v = qkv.split([nh * hd, nkv * hd, nkv * hd], -1)
            q = _rope(q.view(B, T, nh, hd).transpose(1, 2), self.inv, pos)
            k = _rope(k.view(B, T, nkv, hd).transpose(1, 2), self.inv, pos)
            v = v.view(B, T, nkv, hd).transpose(1, 2)
            if nkv != nh:
                k, v = k.repeat_interleave(nh // nkv, 1), v.repeat_interleave(nh // nkv, 1)
            o = F.scaled_dot_product_attention(q.to(self.dtype), k.to(self.dtype), v.to(self.dtype), attn_mask=mask)
            x = x + L["s1"] * lin(o.transpose(1, 2).reshape(B, T, nh * hd), L["o"]).view(B, T, H)
            h = F.layer_norm(x, (H,), *L["ln2"], c.norm_eps)
            m = F.gelu(lin(h, L["fc1"])) if c.hidden_act == "gelu" else F.gelu(lin(h, L["fc1"]), approximate="tanh")
            x = x + L["s2"] * lin(m, L["fc2"]).view(B, T, H)
        return x

    # -- resampling --------------------------------------------------------
    def _downsample(self, x: torch.Tensor) -> torch.Tensor:
        """Causal stride-2 conv with replicate padding; x [B, T, H] -> [B, ceil(T / 2), H]."""
        k = self.down_w.shape[-1]
        stride = 2
        T = x.shape[1]
        total = k - stride
        n_frames = math.ceil((T - k + total) / stride + 1) - 1
        extra = n_frames * stride + k - total - T
        xp = F.pad(x.transpose(1, 2), (total, extra), mode="replicate")
        return F.conv1d(xp, self.down_w, stride=stride).transpose(1, 2)

    def _upsample(self, x: torch.Tensor) -> torch.Tensor:
        """Depthwise transposed conv, stride 2, trimmed causally; [B, T, H] -> [B, 2T, H]."""
        k = self.up_w.shape[-1]
        y = F.conv_transpose1d(x.transpose(1, 2), self.up_w, stride=2, groups=self.cfg.upsample_groups)
        total = k - 2
        right = math.ceil(total * self.cfg.trim_right_ratio)
        return y[..., total - right:y.shape[-1] - right].transpose(1, 2)

    # -- quantiser ---------------------------------------------------------
    @torch.no_grad()
    def quantize(self, z: torch.Tensor, n_q: int) -> torch.Tensor:
        """z [B, T, H] -> codes [B, n_q, T] (semantic stage first)."""
        c = self.cfg
        B, T, H = z.shape
        codes = []
        for gi, g in enumerate(self.groups):
            n = c.num_semantic_quantizers if gi == 0 else n_q - c.num_semantic_quantizers
            if n <= 0:
                continue
            r = z.reshape(B * T, H) @ g["inp"].t()
            for book, sq in zip(g["books"][:n], g["sq"][:n]):
                d = (r.pow(2).sum(1, keepdim=True) - 2 * r @ book.t() + sq[None]).clamp_min(0)
                idx = d.argmin(1)
                r = r - book[idx]
                codes.append(idx.view(B, T))
        return torch.stack(codes, 1)

    @torch.no_grad()
    def dequantize(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, n, T] -> [B, T, H] fp32."""
        c = self.cfg
        codes = codes.to(self.device).long()
        B, n, T = codes.shape
        out = 0
        for gi, g in enumerate(self.groups):
            lo = 0 if gi == 0 else c.num_semantic_quantizers
            hi = c.num_semantic_quantizers if gi == 0 else n
            if hi <= lo:
                continue
            s = sum(g["books"][i - lo][codes[:, i].reshape(-1)] for i in range(lo, hi))
            out = out + s @ g["out"].t()
        return out.view(B, T, -1)

    # -- codec API ---------------------------------------------------------
    @torch.no_grad()
    def encode_latents(self, audio: torch.Tensor) -> torch.Tensor:
        """audio [B, C, samples] -> [B, frames at 12.5 Hz, hidden] fp32 (before quantisation)."""
        x = audio.to(self.device, self.dtype).transpose(1, 2).contiguous()
        h = self.seanet._stack(x, self.seanet.enc).float()
        h = self._transformer(h, "encoder_transformer")
        return self._downsample(h)

    @torch.no_grad()
    def encode(self, audio, num_quantizers: int | None = None) -> torch.Tensor:
        """Mono PCM [samples] / [B, C, samples] at 24 kHz -> codes [B, n_q, frames]."""
        x = torch.as_tensor(audio, dtype=torch.float32)
        while x.dim() < 3:
            x = x[None]
        n_q = self.cfg.num_quantizers if num_quantizers is None else num_quantizers
        return self.quantize(self.encode_latents(x), n_q)

    @torch.no_grad()
    def decode(self, codes: torch.Tensor) -> torch.Tensor:
        """codes [B, n, frames] -> audio [B, C, samples] fp32."""
        h = self._upsample(self.dequantize(codes))
        h = self._transformer(h, "decoder_transformer")
        y = self.seanet._stack(h.to(self.dtype).contiguous(), self.seanet.dec)
        return y.float().transpose(1, 2)
