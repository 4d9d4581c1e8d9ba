"""FLUX.1 text encoders: T5 v1.1 (``text_encoder_2``, per-token context
[512, 4096]) and CLIP ViT-L/14 text (``text_encoder``, pooled [768]), in the HF
``T5EncoderModel`` / ``CLIPTextModel`` tensor layouts.

T5 v1.1: pre-RMSNorm blocks (no mean subtraction, fp32 statistics), attention
without the 1/sqrt(d) scale plus a learned bidirectional relative-position
bias (32 log-spaced buckets up to distance 128, owned by block 0 and shared by
every block), gated GELU (tanh form) feed-forward. FLUX pads the prompt to a
fixed length and passes no attention mask, so pad tokens are attended.

CLIP text: learned absolute positions, pre-LayerNorm blocks with causal
self-attention and quick-GELU MLP, final LayerNorm; the pooled output is the
hidden state at the first end-of-text token (the highest token id for the
original vocabulary).

Both run once per prompt, so they are built from this package's GEMM
(``ops.linear`` on CUDA, bf16) plus torch for the small remaining ops
(attention with T5's additive bias, norms); on CPU everything is fp32 torch.

Reference: crates/rlx-flux1/src/t5.rs (relative_position_bucket, no mask),
src/clip.rs (pooled EOS state).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


def _linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    if x.is_cuda and x.dtype == torch.bfloat16:
        from .. import ops
        y = ops.linear(x.reshape(-1, x.shape[-1]).contiguous(), w, bias=b)
        return y.view(*x.shape[:-1], w.shape[0])
    y = x @ w.t()
    return y + b if b is not None else y


# ---------------------------------------------------------------------------
# T5 v1.1 encoder
# ---------------------------------------------------------------------------

@dataclass
class T5Config:
    vocab_size: int = 32128
    d_model: int = 4096
    d_kv: int = 64
    d_ff: int = 10240
    num_layers: int = 24
    num_heads: int = 64
    relative_attention_num_buckets: int = 32
    relative_attention_max_distance: int = 128
    layer_norm_epsilon: float = 1e-6

    @classmethod
    def from_dict(cls, d: dict) -> "T5Config":
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d})


def relative_position_bucket(rel: torch.Tensor, num_buckets: int, max_distance: int) -> torch.Tensor:
    """Bidirectional bucket of relative position (key - query): half the
    buckets per sign; exact buckets for |rel| < num_buckets / 4, log-spaced
    ones up to max_distance beyond."""
    nb = num_buckets // 2
    out = (rel > 0).long() * nb
    n = rel.abs()
    max_exact = nb // 2
    large = max_exact + (torch.log(n.float() / max_exact + 1e-20) / math.log(max_distance / max_exact)
                         * (nb - max_exact)).long()
    large = torch.clamp(large, max=nb - 1)
    return out + torch.where(n < max_exact, n, large)


def _t5_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (w.float() * y).to(x.dtype)


class T5Encoder:
    def __init__(self, cfg: T5Config, weights, device="cpu", dtype: torch.dtype | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        get = (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        self.embed = dv(get("shared.weight") if "shared.weight" in weights else get("encoder.embed_tokens.weight"))
        self.rel_bias = get("encoder.block.0.layer.0.SelfAttention.relative_attention_bias.weight").to(
            self.device, torch.float32)
        self.blocks = []
        for i in range(cfg.num_layers):
            p = f"encoder.block.{i}.layer."
            blk = dict(ln1=dv(get(p + "0.layer_norm.weight")),
                       qkv=dv(torch.cat([get(p + f"0.SelfAttention.{n}.weight") for n in "qkv"], 0)),
                       o=dv(get(p + "0.SelfAttention.o.weight")), ln2=dv(get(p + "1.layer_norm.weight")),
                       wi=dv(torch.cat([get(p + "1.DenseReluDense.wi_0.weight"),
                                        get(p + "1.DenseReluDense.wi_1.weight")], 0)),
                       wo=dv(get(p + "1.DenseReluDense.wo.weight")))
            self.blocks.append(blk)
        self.final = dv(get("encoder.final_layer_norm.weight"))

    def position_bias(self, L: int) -> torch.Tensor:
        c = self.cfg
        pos = torch.arange(L, device=self.device)
        b = relative_position_bucket(pos[None, :] - pos[:, None], c.relative_attention_num_buckets,
                                     c.relative_attention_max_distance)
        return self.rel_bias[b].permute(2, 0, 1)  # [heads, L, L]

    @torch.no_grad()
    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        """ids [B, L] -> [B, L, d_model] (no attention mask, as FLUX uses it)."""
        c = self.cfg
        ids = ids.to(self.device)
        B, L = ids.shape
        h = self.embed[ids]
        bias = self.position_bias(L).to(self.dtype)
        inner = c.num_heads * c.d_kv
        for blk in self.blocks:
            x = _t5_norm(h, blk["ln1"], c.layer_norm_epsilon)
            q, k, v = _linear(x, blk["qkv"]).split(inner, -1)
            q, k, v = (t.view(B, L, c.num_heads, c.d_kv).transpose(1, 2) for t in (q, k, v))
            a = F.scaled_dot_product_attention(q, k, v, attn_mask=bias.unsqueeze(0).expand(B, -1, -1, -1),
                                               scale=1.0)
            h = h + _linear(a.transpose(1, 2).reshape(B, L, inner), blk["o"])
            x = _t5_norm(h, blk["ln2"], c.layer_norm_epsilon)
            g, u = _linear(x, blk["wi"]).chunk(2, -1)
            h = h + _linear(F.gelu(g, approximate="tanh") * u, blk["wo"])
        return _t5_norm(h, self.final, c.layer_norm_epsilon)


# ---------------------------------------------------------------------------
# CLIP text encoder
# ---------------------------------------------------------------------------

@dataclass
class CLIPTextConfig:
    vocab_size: int = 49408
    hidden_size: int = 768
    intermediate_size: int = 3072
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    max_position_embeddings: int = 77
    layer_norm_eps: float = 1e-5
    eos_token_id: int = 2
    hidden_act: str = "quick_gelu"

    @classmethod
    def from_dict(cls, d: dict) -> "CLIPTextConfig":
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d})


class CLIPTextEncoder:
    def __init__(self, cfg: CLIPTextConfig, weights, device="cpu", dtype: torch.dtype | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        get = (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        p = "text_model."
        self.tok = dv(get(p + "embeddings.token_embedding.weight"))
        self.pos = dv(get(p + "embeddings.position_embedding.weight"))
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            q = f"{p}encoder.layers.{i}."
            a = q + "self_attn."
            self.layers.append(dict(
                ln1=(dv(get(q + "layer_norm1.weight")), dv(get(q + "layer_norm1.bias"))),
                qkv=dv(torch.cat([get(a + f"{n}_proj.weight") for n in "qkv"], 0)),
                qkv_b=dv(torch.cat([get(a + f"{n}_proj.bias") for n in "qkv"], 0)),
                o=(dv(get(a + "out_proj.weight")), dv(get(a + "out_proj.bias"))),
                ln2=(dv(get(q + "layer_norm2.weight")), dv(get(q + "layer_norm2.bias"))),
                fc1=(dv(get(q + "mlp.fc1.weight")), dv(get(q + "mlp.fc1.bias"))),
                fc2=(dv(get(q + "mlp.fc2.weight")), dv(get(q + "mlp.fc2.bias")))))
        self.final = (dv(get(p + "final_layer_norm.weight")), dv(get(p + "final_layer_norm.bias")))

    def _act(self, x):
        if self.cfg.hidden_act == "quick_gelu":
            return x * torch.sigmoid(1.702 * x)
        return F.gelu(x)

    @torch.no_grad()
    def __call__(self, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """ids [B, L] -> (last hidden [B, L, H], pooled [B, H])."""
        c = self.cfg
        ids = ids.to(self.device)
        B, L = ids.shape
        H, nh = c.hidden_size, c.num_attention_heads
        h = self.tok[ids] + self.pos[:L]
        for ly in self.layers:
            x = F.layer_norm(h.float(), (H,), ly["ln1"][0].float(), ly["ln1"][1].float(), c.layer_norm_eps).to(h.dtype)
            q, k, v = _linear(x, ly["qkv"], ly["qkv_b"]).split(H, -1)
            q, k, v = (t.view(B, L, nh, H // nh).transpose(1, 2) for t in (q, k, v))
            a = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            h = h + _linear(a.transpose(1, 2).reshape(B, L, H), *ly["o"])
            x = F.layer_norm(h.float(), (H,), ly["ln2"][0].float(), ly["ln2"][1].float(), c.layer_norm_eps).to(h.dtype)
            h = h + _linear(self._act(_linear(x, *ly["fc1"])), *ly["fc2"])
        h = F.layer_norm(h.float(), (H,), self.final[0].float(), self.final[1].float(), c.layer_norm_eps)
        if c.eos_token_id == 2:  # original CLIP vocabulary: the end-of-text token has the highest id
            eos = ids.argmax(-1)
        else:
            eos = (ids == c.eos_token_id).int().argmax(-1)
        return h, h[torch.arange(B, device=h.device), eos]
