"""Pixtral vision encoder and the Mistral-3 vision-language model (mistral3).

Pixtral tower (images at their own sizes, no resizing to a fixed grid):

    patches  = conv(p x p, stride p, no bias) over the image cropped to a
               multiple of p, computed as one GEMM on the unfolded patches
    x        = rmsnorm(patches) (eps 1e-5)
    RoPE 2-D = for the patch at grid (r, c): the first D/4 rotation pairs turn by
               r * f_even, the next D/4 by c * f_odd (f_m = theta^(-2m / D)),
               half-split rotation
    blocks   = x += attn(rmsnorm(x)); x += W_down(act(W_gate x) * W_up x);
               attention sees only the patches of the same image

Mistral-3 projector: rmsnorm (the text model's eps) -> patch merger (each
s x s block of merged patches, channel-major, through one linear) -> linear_1
-> GELU -> linear_2. The processor writes one image token per merged patch,
with a break token after every row and an end token after the last, so an
image's tokens form one run per grid row; each run is one multimodal segment
of the engine's prompt.

GEMMs run on the package's tcgen05 linear in bf16 on the GPU (fp32 on CPU);
the LM is the package's decoder on the GPU and the fp32 oracle on CPU.

Checkpoint names: transformers' Mistral3ForConditionalGeneration
(``model.vision_tower.*``, ``model.multi_modal_projector.*``,
``model.language_model.*``) or the earlier layout without ``model.``.

Reference: crates/rlx-mistral-vl (Pixtral / Ministral vision encoder,
src/config.rs PixtralVisionConfig, src/encoder.rs); transformers'
Mistral3ForConditionalGeneration is the CPU oracle.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from ..config import DecoderConfig
from .flux_text import _linear
from .llava import _View


@dataclass
class PixtralConfig:
    hidden_size: int = 1024
    intermediate_size: int = 4096
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    head_dim: int = 64
    num_channels: int = 3
    image_size: int = 1024
    patch_size: int = 16
    rope_theta: float = 10000.0
    hidden_act: str = "gelu"

    @classmethod
    def from_dict(cls, d: dict) -> "PixtralConfig":
        kw = {k: d[k] for k in cls.__dataclass_fields__ if k in d and d[k] is not None}
        rp = d.get("rope_parameters") or {}
        if "rope_theta" in rp:
            kw["rope_theta"] = float(rp["rope_theta"])
        kw.setdefault("head_dim", kw.get("hidden_size", cls.hidden_size) // kw.get("num_attention_heads",
                                                                                      cls.num_attention_heads))
        return cls(**kw)


def _act(name: str, x: torch.Tensor) -> torch.Tensor:
    if name == "gelu":
        return F.gelu(x)
    if name in ("gelu_pytorch_tanh", "gelu_new"):
        return F.gelu(x, approximate="tanh")
    if name == "silu":
        return F.silu(x)
    raise NotImplementedError(f"activation {name!r}")


class PixtralEncoder:
    def __init__(self, cfg: PixtralConfig, weights, device="cpu"):
        self.cfg, self.device = cfg, torch.device(device)
        self.dtype = torch.bfloat16 if self.device.type == "cuda" else torch.float32
        get = (lambda k: weights.take(k)) if hasattr(weights, "take") else (lambda k: weights[k])
        dv = lambda n: get(n).to(self.device, self.dtype).contiguous()  # noqa: E731
        f32 = lambda n: get(n).to(self.device, torch.float32)  # noqa: E731
        c = cfg
        self.patch_w = dv("patch_conv.weight").reshape(c.hidden_size, -1).contiguous()  # [(c, kh, kw)]
        self.ln_pre = f32("ln_pre.weight")
        self.layers = []
        for i in range(c.num_hidden_layers):
            p = f"transformer.layers.{i}."
            a = p + "attention."
            self.layers.append(dict(
                n1=f32(p + "attention_norm.weight"), n2=f32(p + "ffn_norm.weight"),
                qkv=torch.cat([dv(a + "q_proj.weight"), dv(a + "k_proj.weight"), dv(a + "v_proj.weight")]),
                o=dv(a + "o_proj.weight"),
                gu=torch.cat([dv(p + "feed_forward.gate_proj.weight"), dv(p + "feed_forward.up_proj.weight")]),
                down=dv(p + "feed_forward.down_proj.weight")))
        D = c.head_dim
        f = c.rope_theta ** (-torch.arange(0, D, 2, dtype=torch.float64) / D)
        self.f_row, self.f_col = f[0::2].float().to(self.device), f[1::2].float().to(self.device)

    @staticmethod
    def _rms(x, w, eps=1e-5):
        x = x.float()
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    def _rope(self, x: torch.Tensor, gh: int, gw: int) -> torch.Tensor:
        r = torch.arange(gh, device=self.device).repeat_interleave(gw).float()
        col = torch.arange(gw, device=self.device).repeat(gh).float()
        ang = torch.cat([r[:, None] * self.f_row[None], col[:, None] * self.f_col[None]], -1)  # [N, D/2]
        cos, sin = ang.cos()[:, None], ang.sin()[:, None]
        h = x.shape[-1] // 2
        x1, x2 = x[..., :h], x[..., h:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)

    @torch.no_grad()
    def hidden_states(self, image: torch.Tensor, layer: int = -1) -> tuple[torch.Tensor, int, int]:
        """One image [3, H, W] -> (hidden state after ``layer`` blocks [N, hidden]
        (HF hidden_states indexing), patch rows, patch columns)."""
        c = self.cfg
        p = c.patch_size
        img = image.to(self.device, torch.float32)
        gh, gw = img.shape[-2] // p, img.shape[-1] // p
        img = img[:, : gh * p, : gw * p]
        patches = img.reshape(c.num_channels, gh, p, gw, p).permute(1, 3, 0, 2, 4).reshape(gh * gw, -1)
        x = self._rms(_linear(patches.to(self.dtype).contiguous(), self.patch_w, None), self.ln_pre)
        n_blocks = layer % (len(self.layers) + 1)
        N, nh, D = x.shape[0], c.num_attention_heads, c.head_dim
        for L in self.layers[:n_blocks]:
            h = self._rms(x, L["n1"]).to(self.dtype)
            q, k, v = _linear(h, L["qkv"], None).float().view(N, 3, nh, D).unbind(1)
            q, k = self._rope(q, gh, gw), self._rope(k, gh, gw)
            o = F.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1),
                                               scale=D ** -0.5)
            x = x + _linear(o.transpose(0, 1).reshape(N, nh * D).to(self.dtype), L["o"], None).float()
            h = self._rms(x, L["n2"]).to(self.dtype)
            gu = _linear(h, L["gu"], None).float()
            I = gu.shape[1] // 2
            y = (_act(c.hidden_act, gu[:, :I]) * gu[:, I:]).to(self.dtype)
            x = x + _linear(y, L["down"], None).float()
        return x, gh, gw


@dataclass
class Mistral3Config:
    vision: PixtralConfig
    text: DecoderConfig
    image_token_index: int = 10
    spatial_merge_size: int = 2
    vision_feature_layer: int = -1
    projector_hidden_act: str = "gelu"

    @classmethod
    def from_dict(cls, d: dict) -> "Mistral3Config":
        tc = dict(d.get("text_config") or {})
        tc.setdefault("model_type", "mistral")
        layer = d.get("vision_feature_layer", -1)
        if isinstance(layer, (list, tuple)):
            raise NotImplementedError("multi-layer vision features (a list of layers) are not supported")
        return cls(vision=PixtralConfig.from_dict(d.get("vision_config") or {}), text=DecoderConfig.from_hf_dict(tc),
                   image_token_index=int(d.get("image_token_index", d.get("image_token_id", 10))),
                   spatial_merge_size=int(d.get("spatial_merge_size", 2)), vision_feature_layer=int(layer),
                   projector_hidden_act=d.get("projector_hidden_act", "gelu"))


class Mistral3VLM:
    def __init__(self, cfg: Mistral3Config, weights, device="cpu", lm=None):
        self.cfg, self.device = cfg, torch.device(device)
        self.vision = PixtralEncoder(cfg.vision, _View(weights, "vision"), device=device)
        pv = _View(weights, "proj")
        dt = self.vision.dtype
        dv = lambda n: pv[n].to(self.device, dt).contiguous() if n in pv else None  # noqa: E731
        self.norm_w = pv["norm.weight"].to(self.device, torch.float32)
        self.merge = dv("patch_merger.merging_layer.weight")
        self.p1 = (dv("linear_1.weight"), dv("linear_1.bias"))
        self.p2 = (dv("linear_2.weight"), dv("linear_2.bias"))
        text = _View(weights, "text")
        if lm is not None:
            self.lm = lm
        elif self.device.type == "cuda":
            from ..registry import build_model
            self.lm = build_model(cfg.text, text, device=self.device)
        else:
            from .oracle import DecoderOracle
            self.lm = DecoderOracle(cfg.text, {k: v.float() for k, v in text.dict().items()}, device=self.device)

    @torch.no_grad()
    def image_tokens(self, image: torch.Tensor) -> tuple[torch.Tensor, int, int]:
        """One preprocessed image [3, H, W] -> (projected tokens [rows * cols, H_text], rows, cols)
        on the merged grid."""
        c = self.cfg
        s = c.spatial_merge_size
        x, gh, gw = self.vision.hidden_states(image, c.vision_feature_layer)
        x = self.vision._rms(x, self.norm_w, c.text.rms_norm_eps)
        d = x.shape[-1]
        grid = F.unfold(x.t().reshape(1, d, gh, gw), kernel_size=s, stride=s)  # [1, d s s, L]
        merged = grid.view(d * s * s, -1).t().to(self.vision.dtype).contiguous()
        h = _linear(merged, self.merge, None)
        h = _act(c.projector_hidden_act, _linear(h, *self.p1).float()).to(h.dtype)
        return _linear(h, *self.p2), gh // s, gw // s

    def placeholder_rows(self, ids: list[int]) -> list[int]:
        return [i for i, t in enumerate(ids) if t == self.cfg.image_token_index]

    @torch.no_grad()
    def mm_segments(self, ids: list[int], images) -> list[tuple[int, torch.Tensor]]:
        """(first position, rows) of every contiguous run of image tokens in ``ids``,
        filled in order with the images' projected tokens (``images``: a list of
        [3, H, W] or a [B, 3, H, W] batch)."""
        feats = torch.cat([self.image_tokens(im)[0] for im in images])
        rows = self.placeholder_rows(ids)
        if len(rows) != feats.shape[0]:
            raise ValueError(f"prompt has {len(rows)} image tokens; the images give {feats.shape[0]}")
        segs, start = [], 0
        for j in range(1, len(rows) + 1):
            if j == len(rows) or rows[j] != rows[j - 1] + 1:
                segs.append((rows[start], feats[start:j]))
                start = j
        return segs

    @torch.no_grad()
    def oracle_logits(self, ids: list[int], images) -> torch.Tensor:
        """fp32 logits [T, V] of the whole prompt (the CPU oracle path)."""
        segs = self.mm_segments(ids, images)
        rows = torch.cat([torch.arange(p, p + e.shape[0]) for p, e in segs])
        emb = torch.cat([e for _, e in segs]).float()
        lg, _ = self.lm.forward(torch.tensor(ids), mm=(rows, emb))
        return lg
