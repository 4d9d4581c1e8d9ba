"""LFM2 hybrid decoder (Liquid AI ``lfm2``): gated short-convolution layers
interleaved with GQA attention layers, SwiGLU feed-forward in every layer.

Short-convolution layer:

    [B | C | x] = in_proj(rmsnorm(h))            (3 x hidden)
    y           = C * conv1d(B * x)               (depthwise, causal, kernel L_cache = 3, no activation)
    h          += out_proj(y)

Attention layers: per-head RMSNorm on q and k (plain weights), RoPE,
out_proj. The feed-forward width follows ``block_auto_adjust_ff_dim``
(2/3 of intermediate_size, times the multiplier, rounded up to
``block_multiple_of``). The final norm is called ``embedding_norm``.

B200 layout: paged KV for the attention layers only; per sequence a state
slot holding each conv layer's window of the last K-1 values of B * x
(double-buffered by position parity). Decode runs the conv step as one
sm_100a kernel per layer (``shortconv_decode_kernel`` in
``csrc/linear_attn/gdn.cu``); prefill runs the depthwise convolution per
sequence in torch. Everything else is the package's GEMM / attention kernels.

Reference: rlx-models-core src/standard_decoder.rs:1353 (`build_lfm2_prefill`)
and the LFM2 family of the reference; transformers ``lfm2`` is the CPU oracle.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field, fields

import torch
import torch.nn.functional as F

from ..ops import rope_inv_freq
from ..runtime.kv_cache import BLOCK_SIZE, PagedKVCache


@dataclass
class Lfm2Config:
    model_type: str = "lfm2"
    vocab_size: int = 65536
    hidden_size: int = 2560
    intermediate_size: int = 12288
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 8
    norm_eps: float = 1e-5
    rope_theta: float = 1e6
    max_position_embeddings: int = 128000
    tie_word_embeddings: bool = True
    conv_bias: bool = False
    conv_L_cache: int = 3
    block_multiple_of: int = 256
    block_ffn_dim_multiplier: float | None = 1.0
    block_auto_adjust_ff_dim: bool = True
    layer_types: list | None = None
    bos_token_id: int | None = 1
    eos_token_id: int | list | None = 2
    extra: dict = field(default_factory=dict)

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def rms_norm_eps(self) -> float:
        return self.norm_eps

    @property
    def ff_dim(self) -> int:
        n = self.intermediate_size
        if self.block_auto_adjust_ff_dim:
            n = int(2 * n / 3)
            if self.block_ffn_dim_multiplier is not None:
                n = int(self.block_ffn_dim_multiplier * n)
                m = self.block_multiple_of
                n = m * ((n + m - 1) // m)
        return n

    def is_attention(self, i: int) -> bool:
        return self.layer_types is None or self.layer_types[i] == "full_attention"

    @classmethod
    def from_dict(cls, d: dict) -> "Lfm2Config":
        kw = {f.name: d[f.name] for f in fields(cls) if f.name in d and f.name != "extra"}
        rp = d.get("rope_parameters") or {}
        if "rope_theta" in rp:
            kw["rope_theta"] = float(rp["rope_theta"])
        if kw.get("layer_types") is None and d.get("full_attn_idxs") is not None:
            idx = set(d["full_attn_idxs"])
            kw["layer_types"] = ["full_attention" if i in idx else "conv" for i in range(d["num_hidden_layers"])]
        return cls(**kw)

    @classmethod
    def from_file(cls, path: str) -> "Lfm2Config":
        with open(os.path.join(path, "config.json") if os.path.isdir(path) else path) as f:
            return cls.from_dict(json.load(f))

    def to_hf_dict(self) -> dict:
        d = {f.name: getattr(self, f.name) for f in fields(self) if f.name != "extra"}
        d["rope_parameters"] = {"rope_type": "default", "rope_theta": self.rope_theta}
        d["full_attn_idxs"] = [i for i in range(self.num_hidden_layers) if self.is_attention(i)]
        return d


def is_lfm2_config(path: str) -> bool:
    p = os.path.join(path, "config.json") if os.path.isdir(path) else path
    try:
        with open(p) as f:
            return json.load(f).get("model_type") == "lfm2"
    except (OSError, ValueError):
        return False


def _getter(weights):
    return (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])


def short_conv(bx: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, window: torch.Tensor | None):
    """bx [H, L] (B * x of one sequence), w [H, K], window [H, K-1] (None =
    zeros). Returns (conv [H, L] in bx's dtype, new window)."""
    K = w.shape[1]
    if window is None:
        window = bx.new_zeros(bx.shape[0], K - 1)
    full = torch.cat([window.to(bx.dtype), bx], 1)
    y = F.conv1d(full[None].float(), w.float()[:, None, :], None if bias is None else bias.float(),
                 groups=bx.shape[0])[0]
    return y.to(bx.dtype), full[:, -(K - 1):]


def random_weights(cfg: Lfm2Config, seed: int = 0, device="cpu", dtype=torch.bfloat16) -> dict:
    gen = torch.Generator(device=device).manual_seed(seed)
    H, I = cfg.hidden_size, cfg.ff_dim
    w = {}

    def lin(name, o, i):
        w[name] = (torch.randn(o, i, generator=gen, device=device) / math.sqrt(i)).to(dtype)

    def vec(name, n):
        w[name] = (1.0 + 0.1 * torch.randn(n, generator=gen, device=device)).to(dtype)

    w["model.embed_tokens.weight"] = torch.randn(cfg.vocab_size, H, generator=gen, device=device).to(dtype)
    vec("model.embedding_norm.weight", H)
    if not cfg.tie_word_embeddings:
        lin("lm_head.weight", cfg.vocab_size, H)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        vec(p + "operator_norm.weight", H)
        vec(p + "ffn_norm.weight", H)
        lin(p + "feed_forward.w1.weight", I, H)
        lin(p + "feed_forward.w3.weight", I, H)
        lin(p + "feed_forward.w2.weight", H, I)
        if cfg.is_attention(i):
            a, D = p + "self_attn.", cfg.head_dim
            lin(a + "q_proj.weight", cfg.num_attention_heads * D, H)
            lin(a + "k_proj.weight", cfg.num_key_value_heads * D, H)
            lin(a + "v_proj.weight", cfg.num_key_value_heads * D, H)
            lin(a + "out_proj.weight", H, cfg.num_attention_heads * D)
            vec(a + "q_layernorm.weight", D)
            vec(a + "k_layernorm.weight", D)
        else:
            a = p + "conv."
            lin(a + "in_proj.weight", 3 * H, H)
            lin(a + "out_proj.weight", H, H)
            w[a + "conv.weight"] = (torch.randn(H, 1, cfg.conv_L_cache, generator=gen, device=device) * 0.5).to(dtype)
    return w


class Lfm2Oracle:
    """fp32 full-sequence forward."""

    def __init__(self, cfg: Lfm2Config, weights, device="cpu"):
        self.cfg, self.device, self.get = cfg, torch.device(device), _getter(weights)
        self.has = lambda n: n in weights  # noqa: E731
        self.inv, self.mult = rope_inv_freq(cfg.head_dim, cfg.rope_theta, None, cfg.max_position_embeddings)

    def _t(self, n):
        return self.get(n).to(self.device, torch.float32)

    def _rms(self, x, n):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.norm_eps) * self._t(n)

    @torch.no_grad()
    def logits(self, ids, mm=None) -> torch.Tensor:
        """``mm`` = (rows, embeds): input embeddings replaced at those rows
        (image tokens of a vision-language prompt)."""
        from ..ops import reference as R
        c = self.cfg
        ids = torch.as_tensor(ids, device=self.device).long()
        S = ids.shape[0]
        pos = torch.arange(S, device=self.device)
        h = self._t("model.embed_tokens.weight")[ids]
        if mm is not None:
            h = h.index_copy(0, mm[0].to(self.device).long(), mm[1].to(self.device, torch.float32))
        nh, nkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            x = self._rms(h, p + "operator_norm.weight")
            if c.is_attention(i):
                a = p + "self_attn."
                q = self._rms((x @ self._t(a + "q_proj.weight").t()).view(S, nh, D), a + "q_layernorm.weight")
                k = self._rms((x @ self._t(a + "k_proj.weight").t()).view(S, nkv, D), a + "k_layernorm.weight")
                v = (x @ self._t(a + "v_proj.weight").t()).view(S, nkv, D)
                q, k = R.rope(q, pos, self.inv, self.mult), R.rope(k, pos, self.inv, self.mult)
                o = R.attention(q, k, v, pos, pos, D ** -0.5, causal=True).reshape(S, nh * D)
                h = h + o @ self._t(a + "out_proj.weight").t()
            else:
                a = p + "conv."
                b_in, b_out, bias = (self._t(a + n) if self.has(a + n) else 0.0
                                     for n in ("in_proj.bias", "out_proj.bias", "conv.bias"))
                Bg, Cg, xx = (x @ self._t(a + "in_proj.weight").t() + b_in).chunk(3, -1)
                y, _ = short_conv((Bg * xx).t(), self._t(a + "conv.weight")[:, 0],
                                  bias if torch.is_tensor(bias) else None, None)
                h = h + (Cg * y.t()) @ self._t(a + "out_proj.weight").t() + b_out
            x = self._rms(h, p + "ffn_norm.weight")
            f = p + "feed_forward."
            h = h + (F.silu(x @ self._t(f + "w1.weight").t()) * (x @ self._t(f + "w3.weight").t())) \
                @ self._t(f + "w2.weight").t()
        h = self._rms(h, "model.embedding_norm.weight")
        head = "model.embed_tokens.weight" if c.tie_word_embeddings else "lm_head.weight"
        return h @ self._t(head).t()


# ---------------------------------------------------------------------------
# GPU model (engine interface)
# ---------------------------------------------------------------------------

class ConvStateCache:
    """Paged KV for the attention layers + conv windows [n_conv, slots, 2, H, K-1]."""

    def __init__(self, cfg: Lfm2Config, num_blocks: int, num_slots: int, device):
        n_attn = sum(cfg.is_attention(i) for i in range(cfg.num_hidden_layers))
        self.paged = PagedKVCache(max(1, n_attn), num_blocks, cfg.num_key_value_heads, cfg.head_dim, device)
        self.k, self.v = self.paged.k, self.paged.v
        self.num_slots = num_slots
        self.conv = torch.zeros(cfg.num_hidden_layers - n_attn, num_slots, 2, cfg.hidden_size, cfg.conv_L_cache - 1,
                                dtype=torch.bfloat16, device=device)

    def layer(self, i: int):
        return self.paged.layer(i)


class _Layer:
    __slots__ = ("ln1", "ln2", "w_gu", "wd", "wo", "bo", "attn", "idx", "wqkv", "q_norm", "k_norm", "w_in", "b_in",
                 "conv_w", "conv_b")


class Lfm2LM:
    stateful = True

    def __init__(self, cfg: Lfm2Config, weights, device="cuda"):
        from .. import ops
        self.cfg, self.device = cfg, torch.device(device)
        c, dev, bf = cfg, self.device, torch.bfloat16
        self.hkv, self.D = c.num_key_value_heads, c.head_dim
        self.scale = c.head_dim ** -0.5
        inv, self.rope_mult = rope_inv_freq(c.head_dim, c.rope_theta, None, c.max_position_embeddings)
        self.inv_freq = inv.to(dev)
        get = _getter(weights)

        def g(n):
            return get(n).to(dev)

        def dv(t):
            return t.to(dev, bf).contiguous()

        self.embed = dv(g("model.embed_tokens.weight"))
        self.norm = dv(g("model.embedding_norm.weight"))
        self.lm_head = self.embed if c.tie_word_embeddings else dv(g("lm_head.weight"))
        self.layers, n_attn, n_conv = [], 0, 0
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            L = _Layer()
            L.ln1, L.ln2 = dv(g(p + "operator_norm.weight")), dv(g(p + "ffn_norm.weight"))
            f = p + "feed_forward."
            L.w_gu = dv(ops.interleave_gate_up(g(f + "w1.weight"), g(f + "w3.weight")))
            L.wd = dv(g(f + "w2.weight"))
            L.attn = c.is_attention(i)
            L.bo = L.b_in = None
            if L.attn:
                a = p + "self_attn."
                L.idx, n_attn = n_attn, n_attn + 1
                L.wqkv = dv(torch.cat([g(a + "q_proj.weight"), g(a + "k_proj.weight"), g(a + "v_proj.weight")], 0))
                L.q_norm, L.k_norm = dv(g(a + "q_layernorm.weight")), dv(g(a + "k_layernorm.weight"))
                L.wo = dv(g(a + "out_proj.weight"))
            else:
                a = p + "conv."
                L.idx, n_conv = n_conv, n_conv + 1
                L.w_in = dv(g(a + "in_proj.weight"))
                L.conv_w = g(a + "conv.weight").float().reshape(c.hidden_size, -1).contiguous()
                L.conv_b = g(a + "conv.bias").float().contiguous() if (a + "conv.bias") in weights else None
                L.wo = dv(g(a + "out_proj.weight"))
                if (a + "in_proj.bias") in weights:  # conv_bias also puts biases on in_proj / out_proj
                    L.b_in, L.bo = dv(g(a + "in_proj.bias")), dv(g(a + "out_proj.bias"))
            self.layers.append(L)
        self.n_attn = n_attn

    def make_kv_cache(self, num_blocks: int, num_slots: int = 8) -> ConvStateCache:
        return ConvStateCache(self.cfg, num_blocks, num_slots, self.device)

    def kv_bytes_per_block(self) -> int:
        return 2 * max(1, self.n_attn) * self.hkv * BLOCK_SIZE * self.D * 2

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        from .. import ops
        return ops.linear(x, self.lm_head, out_dtype=torch.float32)

    def forward(self, fb, kv: ConvStateCache) -> torch.Tensor:
        x = self.forward_hidden(fb, kv)
        if fb.logit_rows is not None:
            x = x.index_select(0, fb.logit_rows)
        return self.logits(x)

    def _attention(self, L: _Layer, x, fb, kv):
        from .. import ops
        c = self.cfg
        T = x.shape[0]
        kc, vc = kv.layer(L.idx)
        q = ops.qkv_rope(ops.linear(x, L.wqkv), num_q_heads=c.num_attention_heads, num_kv_heads=c.num_key_value_heads,
                         head_dim=c.head_dim, positions=fb.positions, inv_freq=self.inv_freq,
                         rope_scale=self.rope_mult, q_norm=L.q_norm, k_norm=L.k_norm, eps=c.norm_eps, slots=fb.slots,
                         k_cache=kc, v_cache=vc)
        o = torch.empty_like(q)
        nd = fb.num_decode
        if nd > 0:
            ops.decode_attention(q[:nd], kc, vc, fb.dec_block_tables, fb.dec_ctx_lens, scale=self.scale, out=o[:nd])
        if T > nd:
            ops.prefill_attention(q[nd:], kc, vc, fb.pre_block_tables, fb.pre_ctx_lens, fb.pre_cu_q, fb.pre_max_q,
                                  scale=self.scale, out=o[nd:])
        return o.view(T, -1)

    def _conv(self, L: _Layer, x, fb, kv, slots):
        from .. import ops
        from ..ops._ext import ext
        H = self.cfg.hidden_size
        T = x.shape[0]
        p = ops.linear(x, L.w_in, bias=L.b_in)  # [T, B | C | x]
        out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
        nd = fb.num_decode
        if nd > 0:
            ext().shortconv_decode(p[:nd], L.conv_w, L.conv_b, kv.conv[L.idx], slots[:nd], fb.positions[:nd],
                                   out[:nd])
            ops._count(1)
        if T > nd:
            cu, ctx, sl = fb.pre_cu_q.tolist(), fb.pre_ctx_lens.tolist(), slots[nd:].tolist()
            for s, n_ctx in enumerate(ctx):
                a, b = nd + cu[s], nd + cu[s + 1]
                n = b - a
                start, slot = n_ctx - n, sl[s]
                rows = p[a:b]
                bx = (rows[:, :H].float() * rows[:, 2 * H:].float()).to(torch.bfloat16)
                win = kv.conv[L.idx, slot, start & 1] if start > 0 else None
                y, new_win = short_conv(bx.t(), L.conv_w, L.conv_b, win)
                kv.conv[L.idx, slot, (start + n) & 1] = new_win
                out[a:b] = (rows[:, H:2 * H].float() * y.t().float()).to(torch.bfloat16)
        return out

    def forward_hidden(self, fb, kv: ConvStateCache) -> torch.Tensor:
        from .. import ops
        from .decoder import LocalComm
        c = self.cfg
        comm = LocalComm(c.norm_eps)
        slots = fb.seq_slots
        if slots is None:
            nseq = fb.num_decode + (0 if fb.pre_ctx_lens is None else fb.pre_ctx_lens.shape[0])
            slots = torch.arange(nseq, dtype=torch.int32, device=self.device)
        h = ops.embedding(fb.input_ids, self.embed)
        if getattr(fb, "mm_rows", None) is not None:  # image tokens of a vision-language prompt
            h.index_copy_(0, fb.mm_rows, fb.mm_embeds.to(h.dtype))
        x = ops.rmsnorm(h, self.layers[0].ln1, c.norm_eps)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            a = self._attention(L, x, fb, kv) if L.attn else self._conv(L, x, fb, kv, slots)
            x = comm.rowpar_add_norm(a, L.wo, h, L.ln2, bias=L.bo)
            if x.shape[0] <= ops.ACC_MAX_M:
                gu = ops.swiglu_acc(ops.linear_acc(x, L.w_gu))
            else:
                gu = ops.linear_swiglu(x, L.w_gu)
            x = comm.rowpar_add_norm(gu, L.wd, h, self.layers[i + 1].ln1 if i + 1 < n else self.norm)
        return x
