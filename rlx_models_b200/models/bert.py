"""BERT-family text encoders for embeddings (HF ``BertModel`` layout):
word + position + token-type embeddings with LayerNorm, post-LayerNorm
blocks (self-attention with biases, GELU MLP), and pooling into one vector
per text (CLS, mean over non-padding tokens, or the pooler's tanh dense).

Runs on the package's GEMM (``ops.linear``, bf16) on CUDA and in fp32 torch
on CPU; attention uses the padding mask of each batch.

``NomicBertEncoder`` is the NomicBERT variant (transformers ``nomic_bert``
layout): word + token-type embeddings only, rotary positions in every
attention layer, bias-free q / k / v / o, a SwiGLU MLP, and post-LayerNorm
after each sublayer.

Reference: crates/rlx-models-core src/config.rs:30-150 (`BertConfig`,
`NomicBertConfig`) and the embedding families (MODELS.md: 5 embedding
models).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from .flux_text import _linear


@dataclass
class BertConfig:
    vocab_size: int = 30522
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    max_position_embeddings: int = 512
    type_vocab_size: int = 2
    layer_norm_eps: float = 1e-12
    hidden_act: str = "gelu"

    @classmethod
    def from_dict(cls, d: dict) -> "BertConfig":
        return cls(**{k: d[k] for k in cls.__dataclass_fields__ if k in d})


class BertEncoder:
    def __init__(self, cfg: BertConfig, weights, device="cpu", dtype: torch.dtype | None = None, prefix=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        names = list(weights.keys())
        if prefix is None:  # BertModel ("embeddings...") or a task model ("bert.embeddings...")
            prefix = "bert." if any(n.startswith("bert.") for n in names) else ""
        get = (lambda n: weights.take(prefix + n)) if hasattr(weights, "take") else (lambda n: weights[prefix + n])
        has = lambda n: (prefix + n) in weights  # noqa: E731
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        e = "embeddings."
        self.word = dv(get(e + "word_embeddings.weight"))
        self.pos = dv(get(e + "position_embeddings.weight"))
        self.tt = dv(get(e + "token_type_embeddings.weight")) if has(e + "token_type_embeddings.weight") else None
        self.emb_ln = (dv(get(e + "LayerNorm.weight")), dv(get(e + "LayerNorm.bias")))
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"encoder.layer.{i}."
            a = p + "attention."
            self.layers.append(dict(
                qkv=dv(torch.cat([get(a + f"self.{n}.weight") for n in ("query", "key", "value")], 0)),
                qkv_b=dv(torch.cat([get(a + f"self.{n}.bias") for n in ("query", "key", "value")], 0)),
                o=(dv(get(a + "output.dense.weight")), dv(get(a + "output.dense.bias"))),
                ln1=(dv(get(a + "output.LayerNorm.weight")), dv(get(a + "output.LayerNorm.bias"))),
                fc1=(dv(get(p + "intermediate.dense.weight")), dv(get(p + "intermediate.dense.bias"))),
                fc2=(dv(get(p + "output.dense.weight")), dv(get(p + "output.dense.bias"))),
                ln2=(dv(get(p + "output.LayerNorm.weight")), dv(get(p + "output.LayerNorm.bias")))))
        self.pooler = (dv(get("pooler.dense.weight")), dv(get("pooler.dense.bias"))) if has("pooler.dense.weight") \
            else None

    def _ln(self, x, p):
        return F.layer_norm(x.float(), (x.shape[-1],), p[0].float(), p[1].float(), self.cfg.layer_norm_eps).to(x.dtype)

    @torch.no_grad()
    def __call__(self, ids: torch.Tensor, attention_mask: torch.Tensor | None = None,
                 token_type_ids: torch.Tensor | None = None) -> torch.Tensor:
        """ids [B, L] -> last hidden states [B, L, H]."""
        c = self.cfg
        ids = ids.to(self.device)
        B, L = ids.shape
        H, nh = c.hidden_size, c.num_attention_heads
        x = self.word[ids] + self.pos[:L]
        if self.tt is not None:
            tt = token_type_ids.to(self.device) if token_type_ids is not None else torch.zeros_like(ids)
            x = x + self.tt[tt]
        x = self._ln(x, self.emb_ln)
        mask = None
        if attention_mask is not None:
            keep = attention_mask.to(self.device).bool()
            mask = keep[:, None, None, :]  # [B, 1, 1, L]
        for ly in self.layers:
            q, k, v = _linear(x, ly["qkv"], ly["qkv_b"]).split(H, -1)
            q, k, v = (t.view(B, L, nh, H // nh).transpose(1, 2) for t in (q, k, v))
            a = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
            x = self._ln(x + _linear(a.transpose(1, 2).reshape(B, L, H), *ly["o"]), ly["ln1"])
            h = F.gelu(_linear(x, *ly["fc1"]).float()).to(x.dtype)
            x = self._ln(x + _linear(h, *ly["fc2"]), ly["ln2"])
        return x

    def embed(self, ids: torch.Tensor, attention_mask: torch.Tensor | None = None, pooling: str = "mean",
              normalize: bool = True) -> torch.Tensor:
        """[B, H] fp32 sentence embeddings: "cls", "mean" (over non-padding
        tokens) or "pooler" (tanh dense on CLS)."""
        h = self(ids, attention_mask).float()
        if pooling == "cls":
            e = h[:, 0]
        elif pooling == "pooler":
            if self.pooler is None:
                raise ValueError("this checkpoint has no pooler")
            e = torch.tanh(h[:, 0] @ self.pooler[0].float().t() + self.pooler[1].float())
        else:
            m = (attention_mask.to(h.device).float() if attention_mask is not None
                 else torch.ones(h.shape[:2], device=h.device))
            e = (h * m[..., None]).sum(1) / m.sum(1, keepdim=True).clamp_min(1.0)
        return F.normalize(e, dim=-1) if normalize else e


@dataclass
class NomicBertConfig:
    vocab_size: int = 30528
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    type_vocab_size: int = 2
    layer_norm_eps: float = 1e-12
    rope_theta: float = 1000.0

    @classmethod
    def from_dict(cls, d: dict) -> "NomicBertConfig":
        kw = {k: d[k] for k in cls.__dataclass_fields__ if k in d}
        rp = d.get("rope_parameters") or {}
        if "rope_theta" in rp:
            kw["rope_theta"] = float(rp["rope_theta"])
        return cls(**kw)


class NomicBertEncoder(BertEncoder):
    """NomicBERT (``nomic_bert``): rotary attention, SwiGLU MLP, post-norms."""

    def __init__(self, cfg: NomicBertConfig, weights, device="cpu", dtype: torch.dtype | None = None, prefix=None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype or (torch.bfloat16 if self.device.type == "cuda" else torch.float32)
        names = list(weights.keys())
        if prefix is None:
            prefix = "model." if any(n.startswith("model.") for n in names) else ""
        get = (lambda n: weights.take(prefix + n)) if hasattr(weights, "take") else (lambda n: weights[prefix + n])
        has = lambda n: (prefix + n) in weights  # noqa: E731
        dv = lambda t: t.to(self.device, self.dtype).contiguous()  # noqa: E731
        e = "embeddings."
        self.word = dv(get(e + "word_embeddings.weight"))
        self.pos = None
        self.tt = dv(get(e + "token_type_embeddings.weight")) if has(e + "token_type_embeddings.weight") else None
        self.emb_ln = (dv(get(e + "LayerNorm.weight")), dv(get(e + "LayerNorm.bias")))
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"layers.{i}."
            a = p + "self_attn."
            self.layers.append(dict(
                qkv=dv(torch.cat([get(a + f"{n}_proj.weight") for n in "qkv"], 0)),
                o=dv(get(a + "o_proj.weight")),
                ln1=(dv(get(p + "post_attention_layernorm.weight")), dv(get(p + "post_attention_layernorm.bias"))),
                gate=dv(get(p + "mlp.gate_proj.weight")), up=dv(get(p + "mlp.up_proj.weight")),
                down=dv(get(p + "mlp.down_proj.weight")),
                ln2=(dv(get(p + "post_mlp_layernorm.weight")), dv(get(p + "post_mlp_layernorm.bias")))))
        self.pooler = (dv(get("pooler.dense.weight")), dv(get("pooler.dense.bias"))) if has("pooler.dense.weight") \
            else None
        D = cfg.hidden_size // cfg.num_attention_heads
        self.inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, D, 2, dtype=torch.float32) / D))

    @torch.no_grad()
    def __call__(self, ids: torch.Tensor, attention_mask: torch.Tensor | None = None,
                 token_type_ids: torch.Tensor | None = None) -> torch.Tensor:
        from ..ops import reference as R
        c = self.cfg
        ids = ids.to(self.device)
        B, L = ids.shape
        H, nh = c.hidden_size, c.num_attention_heads
        D = H // nh
        x = self.word[ids]
        if self.tt is not None:
            tt = token_type_ids.to(self.device) if token_type_ids is not None else torch.zeros_like(ids)
            x = x + self.tt[tt]
        x = self._ln(x, self.emb_ln)
        mask = attention_mask.to(self.device).bool()[:, None, None, :] if attention_mask is not None else None
        pos = torch.arange(L, device=self.device)
        inv = self.inv_freq.to(self.device)
        for ly in self.layers:
            q, k, v = _linear(x, ly["qkv"]).split(H, -1)
            q, k = (R.rope(t.reshape(B * L, nh, D), pos.repeat(B), inv).reshape(B, L, nh, D).to(x.dtype)
                    for t in (q, k))
            q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.view(B, L, nh, D).transpose(1, 2)
            a = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
            x = self._ln(x + _linear(a.transpose(1, 2).reshape(B, L, H), ly["o"]), ly["ln1"])
            m = F.silu(_linear(x, ly["gate"]).float()) * _linear(x, ly["up"]).float()
            x = self._ln(x + _linear(m.to(x.dtype), ly["down"]), ly["ln2"])
        return x
