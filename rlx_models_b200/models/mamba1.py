"""Mamba-1 (selective SSM) models: ``mamba``, ``falcon_mamba`` and ``jamba``
(Mamba-1 layers + attention layers without positional encoding + top-2 MoE
feed-forward on alternate layers).

Mamba-1 mixer (inner width Di, state N, dt rank R):

    [x | z] = in_proj(norm(h))
    x       = silu(conv1d(x) + bias)                          (kernel 4, causal, depthwise)
    [dt | B | C] = x_proj(x)    (Jamba: RMSNorm on each; Falcon-Mamba: weightless RMSNorm)
    dt      = softplus(dt_proj(dt) + dt_bias)                 [Di]
    h[d, n] = exp(dt[d] A[d, n]) h[d, n] + dt[d] B[n] x[d],   A = -exp(A_log)
    y       = (h C + D x) * silu(z);   out = out_proj(y)

The decay is per (channel, state), so the recurrence is a selective scan
rather than a decayed linear attention. On the GPU one kernel runs the conv
(a channel's K-1 window in registers) and one the scan (a channel's N states
in registers), both over the step's tokens grouped by sequence, prefill and
decode alike; the in / x / dt projections are tcgen05 GEMMs in between.
Per-sequence state slots hold the conv windows and the states.

Reference: crates/rlx-mamba (Mamba-1 selective scan / mamba1_step), crates
rlx-jamba, crates rlx-ssm; transformers ``mamba`` / ``falcon_mamba`` /
``jamba`` are the CPU oracles.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field, fields

import torch
import torch.nn.functional as F

from ..runtime.kv_cache import BLOCK_SIZE, PagedKVCache

MAMBA1_TYPES = ("mamba", "falcon_mamba", "jamba")


@dataclass
class Mamba1Config:
    model_type: str = "mamba"
    vocab_size: int = 50280
    hidden_size: int = 768
    num_hidden_layers: int = 24
    state_size: int = 16
    expand: int = 2
    conv_kernel: int = 4
    time_step_rank: int = 48
    use_conv_bias: bool = True
    rms_norm_eps: float = 1e-5
    mixer_rms_eps: float = 1e-6
    tie_word_embeddings: bool = True
    # jamba
    num_attention_heads: int = 0
    num_key_value_heads: int = 0
    intermediate_size: int = 0
    attn_layer_period: int = 8
    attn_layer_offset: int = 4
    expert_layer_period: int = 2
    expert_layer_offset: int = 1
    num_experts: int = 0
    num_experts_per_tok: int = 2
    max_position_embeddings: int = 262144
    bos_token_id: int | None = None
    eos_token_id: int | list | None = None
    extra: dict = field(default_factory=dict)

    @property
    def inner(self) -> int:
        return self.expand * self.hidden_size

    @property
    def head_dim(self) -> int:
        return self.hidden_size // max(1, self.num_attention_heads)

    def is_attention(self, i: int) -> bool:
        return self.model_type == "jamba" and i % self.attn_layer_period == self.attn_layer_offset

    def is_moe(self, i: int) -> bool:
        return (self.model_type == "jamba" and self.num_experts > 1
                and i % self.expert_layer_period == self.expert_layer_offset)

    @classmethod
    def from_dict(cls, d: dict) -> "Mamba1Config":
        d = dict(d)
        mt = d.get("model_type", "mamba")
        kw = {f.name: d[f.name] for f in fields(cls) if f.name in d and f.name != "extra"}
        if mt == "jamba":
            kw["state_size"] = d.get("mamba_d_state", 16)
            kw["expand"] = d.get("mamba_expand", 2)
            kw["conv_kernel"] = d.get("mamba_d_conv", 4)
            kw["use_conv_bias"] = d.get("mamba_conv_bias", True)
            kw["rms_norm_eps"] = d.get("rms_norm_eps", 1e-6)
            r = d.get("mamba_dt_rank", "auto")
            kw["time_step_rank"] = math.ceil(d["hidden_size"] / 16) if r == "auto" else int(r)
            kw["tie_word_embeddings"] = d.get("tie_word_embeddings", False)
        else:
            kw["rms_norm_eps"] = d.get("layer_norm_epsilon", 1e-5)
            r = d.get("time_step_rank", "auto")
            kw["time_step_rank"] = math.ceil(d["hidden_size"] / 16) if r == "auto" else int(r)
        return cls(**kw)

    @classmethod
    def from_file(cls, path: str) -> "Mamba1Config":
        with open(os.path.join(path, "config.json") if os.path.isdir(path) else path) as f:
            return cls.from_dict(json.load(f))


def is_mamba1_config(path: str) -> bool:
    p = os.path.join(path, "config.json") if os.path.isdir(path) else path
    try:
        with open(p) as f:
            return json.load(f).get("model_type") in MAMBA1_TYPES
    except (OSError, ValueError):
        return False


def _names(cfg: Mamba1Config):
    if cfg.model_type == "jamba":
        return "model.embed_tokens.weight", "model.final_layernorm.weight", "model.layers.{i}.", \
            "input_layernorm", "mamba."
    return "backbone.embeddings.weight", "backbone.norm_f.weight", "backbone.layers.{i}.", "norm", "mixer."


def _getter(weights):
    return (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])


def _rms(x, w, eps):
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y * w if w is not None else y


def selective_scan(x, dt, A, B, C, D, z, state=None):
    """Reference scan for one sequence: x, dt, z [L, Di] fp32 (dt after
    softplus), A [Di, N], B, C [L, N], D [Di]. Returns (y [L, Di], state)."""
    L, Di = x.shape
    h = torch.zeros(Di, A.shape[1], dtype=torch.float32, device=x.device) if state is None else state.float()
    ys = []
    for t in range(L):
        h = torch.exp(dt[t, :, None] * A) * h + dt[t, :, None] * B[t][None, :] * x[t, :, None]
        ys.append(h @ C[t] + D * x[t])
    return torch.stack(ys) * F.silu(z), h


class _Prefixed:
    """Names under ``<prefix>.`` seen with the prefix ``mlp.`` replaced, so
    ``expert_weights`` (which reads ``<layer>mlp.experts...``) finds Jamba's
    ``feed_forward.experts...``."""

    def __init__(self, get, has, prefix: str):
        self.get, self.has, self.prefix = get, has, prefix

    def _real(self, n):
        return self.prefix + n[len("mlp"):] if n.startswith("mlp.") else n

    def __contains__(self, n):
        return self.has(self._real(n))

    def __getitem__(self, n):
        return self.get(self._real(n))


class Mamba1Oracle:
    """fp32 full-sequence forward."""

    def __init__(self, cfg: Mamba1Config, weights, device="cpu"):
        self.cfg, self.device, self.get = cfg, torch.device(device), _getter(weights)
        self.has = lambda n: n in weights  # noqa: E731

    def _t(self, n):
        return self.get(n).to(self.device, torch.float32)

    def mixer(self, m: str, x: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        Di, N, R = c.inner, c.state_size, c.time_step_rank
        xz = x @ self._t(m + "in_proj.weight").t()
        xs, z = xz[:, :Di], xz[:, Di:]
        w = self._t(m + "conv1d.weight")[:, 0]
        b = self._t(m + "conv1d.bias") if self.has(m + "conv1d.bias") else None
        full = torch.cat([xs.new_zeros(c.conv_kernel - 1, Di), xs], 0).t()
        xs = F.silu(F.conv1d(full[None], w[:, None, :], b, groups=Di)[0]).t()
        p = xs @ self._t(m + "x_proj.weight").t()
        dt, B, C = p[:, :R], p[:, R:R + N], p[:, R + N:]
        if c.model_type == "jamba":
            dt = _rms(dt, self._t(m + "dt_layernorm.weight"), c.rms_norm_eps)
            B = _rms(B, self._t(m + "b_layernorm.weight"), c.rms_norm_eps)
            C = _rms(C, self._t(m + "c_layernorm.weight"), c.rms_norm_eps)
        elif c.model_type == "falcon_mamba":
            dt, B, C = (_rms(t, None, c.mixer_rms_eps) for t in (dt, B, C))
        dt = F.softplus(dt @ self._t(m + "dt_proj.weight").t() + self._t(m + "dt_proj.bias"))
        y, _ = selective_scan(xs, dt, -self._t(m + "A_log").exp(), B, C, self._t(m + "D"), z)
        return y @ self._t(m + "out_proj.weight").t()

    @torch.no_grad()
    def logits(self, ids) -> torch.Tensor:
        from ..ops import reference as R
        c = self.cfg
        emb, fin, lay, bn, mix = _names(c)
        ids = torch.as_tensor(ids, device=self.device).long()
        S = ids.shape[0]
        pos = torch.arange(S, device=self.device)
        h = self._t(emb)[ids]
        for i in range(c.num_hidden_layers):
            p = lay.format(i=i)
            x = _rms(h, self._t(p + bn + ".weight"), c.rms_norm_eps)
            if c.is_attention(i):
                a, nh, nkv, D = p + "self_attn.", c.num_attention_heads, c.num_key_value_heads, c.head_dim
                q = (x @ self._t(a + "q_proj.weight").t()).view(S, nh, D)
                k = (x @ self._t(a + "k_proj.weight").t()).view(S, nkv, D)
                v = (x @ self._t(a + "v_proj.weight").t()).view(S, nkv, D)
                o = R.attention(q, k, v, pos, pos, D ** -0.5, causal=True).reshape(S, nh * D)
                h = h + o @ self._t(a + "o_proj.weight").t()
            else:
                h = h + self.mixer(p + mix, x)
            if c.model_type != "jamba":
                continue
            x = _rms(h, self._t(p + "pre_ff_layernorm.weight"), c.rms_norm_eps)
            f = p + "feed_forward."
            if c.is_moe(i):
                from .deepseek import expert_weights
                probs = (x @ self._t(f + "router.weight").t()).softmax(-1)
                top, idx = probs.topk(c.num_experts_per_tok, -1)
                out = torch.zeros_like(x)
                src = _Prefixed(self.get, self.has, p[:-1] + ".feed_forward")
                for e in idx.unique().tolist():
                    rows, slot = (idx == e).nonzero(as_tuple=True)
                    g, u, d = (t.to(self.device, torch.float32) for t in
                               expert_weights(src, "", e, c.intermediate_size))
                    xe = x[rows]
                    out.index_add_(0, rows, ((F.silu(xe @ g.t()) * (xe @ u.t())) @ d.t()) * top[rows, slot, None])
                h = h + out
            else:
                h = h + (F.silu(x @ self._t(f + "gate_proj.weight").t()) * (x @ self._t(f + "up_proj.weight").t())) \
                    @ self._t(f + "down_proj.weight").t()
        h = _rms(h, self._t(fin), c.rms_norm_eps)
        head = emb if c.tie_word_embeddings else "lm_head.weight"
        return h @ self._t(head).t()


def random_weights(cfg: Mamba1Config, seed: int = 0, device="cpu", dtype=torch.bfloat16) -> dict:
    gen = torch.Generator(device=device).manual_seed(seed)
    H, Di, N, R = cfg.hidden_size, cfg.inner, cfg.state_size, cfg.time_step_rank
    emb, fin, lay, bn, mix = _names(cfg)
    w = {}

    def lin(name, o, i):
        w[name] = (torch.randn(o, i, generator=gen, device=device) / math.sqrt(i)).to(dtype)

    def vec(name, n, base=1.0, s=0.1):
        w[name] = (base + s * torch.randn(n, generator=gen, device=device)).to(dtype)

    w[emb] = torch.randn(cfg.vocab_size, H, generator=gen, device=device).to(dtype)
    vec(fin, H)
    if not cfg.tie_word_embeddings:
        lin("lm_head.weight", cfg.vocab_size, H)
    for i in range(cfg.num_hidden_layers):
        p = lay.format(i=i)
        vec(p + bn + ".weight", H)
        if cfg.is_attention(i):
            a, D = p + "self_attn.", cfg.head_dim
            lin(a + "q_proj.weight", cfg.num_attention_heads * D, H)
            lin(a + "k_proj.weight", cfg.num_key_value_heads * D, H)
            lin(a + "v_proj.weight", cfg.num_key_value_heads * D, H)
            lin(a + "o_proj.weight", H, cfg.num_attention_heads * D)
        else:
            m = p + mix
            lin(m + "in_proj.weight", 2 * Di, H)
            w[m + "conv1d.weight"] = (torch.randn(Di, 1, cfg.conv_kernel, generator=gen, device=device) * 0.5).to(dtype)
            vec(m + "conv1d.bias", Di, base=0.0)
            lin(m + "x_proj.weight", R + 2 * N, Di)
            lin(m + "dt_proj.weight", Di, R)
            vec(m + "dt_proj.bias", Di, base=-2.0, s=0.5)
            w[m + "A_log"] = torch.arange(1, N + 1, device=device).float().log().repeat(Di, 1).to(dtype)
            vec(m + "D", Di)
            lin(m + "out_proj.weight", H, Di)
            if cfg.model_type == "jamba":
                vec(m + "dt_layernorm.weight", R)
                vec(m + "b_layernorm.weight", N)
                vec(m + "c_layernorm.weight", N)
        if cfg.model_type == "jamba":
            vec(p + "pre_ff_layernorm.weight", H)
            f, I = p + "feed_forward.", cfg.intermediate_size
            if cfg.is_moe(i):
                lin(f + "router.weight", cfg.num_experts, H)
                for e in range(cfg.num_experts):
                    lin(f + f"experts.{e}.gate_proj.weight", I, H)
                    lin(f + f"experts.{e}.up_proj.weight", I, H)
                    lin(f + f"experts.{e}.down_proj.weight", H, I)
            else:
                lin(f + "gate_proj.weight", I, H)
                lin(f + "up_proj.weight", I, H)
                lin(f + "down_proj.weight", H, I)
    return w


# ---------------------------------------------------------------------------
# GPU model (engine interface)
# ---------------------------------------------------------------------------

class Mamba1Cache:
    """Paged KV for attention layers + per-slot conv windows [n, slots, Di, K-1]
    and SSM states [n, slots, Di, N]."""

    def __init__(self, cfg: Mamba1Config, num_blocks: int, num_slots: int, device):
        n_attn = sum(cfg.is_attention(i) for i in range(cfg.num_hidden_layers))
        n_ssm = cfg.num_hidden_layers - n_attn
        hkv, D = (cfg.num_key_value_heads, cfg.head_dim) if n_attn else (1, 64)
        self.paged = PagedKVCache(max(1, n_attn), num_blocks if n_attn else 1, hkv, D, device)
        self.k, self.v = self.paged.k, self.paged.v
        self.num_slots = num_slots
        self.conv = torch.zeros(n_ssm, num_slots, cfg.inner, cfg.conv_kernel - 1, dtype=torch.bfloat16, device=device)
        self.ssm = torch.zeros(n_ssm, num_slots, cfg.inner, cfg.state_size, dtype=torch.float32, device=device)

    def layer(self, i: int):
        return self.paged.layer(i)


class _Layer:
    __slots__ = ("ln1", "ln2", "attn", "idx", "wqkv", "wo", "w_in", "conv_w", "conv_b", "w_x", "w_dt", "dt_bias",
                 "A_log", "Dp", "n_dt", "n_b", "n_c", "w_gu", "wd", "moe")


class Mamba1LM:
    stateful = True

    def __init__(self, cfg: Mamba1Config, weights, device="cuda"):
        from .. import ops
        from .moe import pack_experts
        self.cfg, self.device = cfg, torch.device(device)
        c, dev, bf = cfg, self.device, torch.bfloat16
        self.hkv = c.num_key_value_heads or 1
        self.D = c.head_dim if c.num_attention_heads else 64
        self.scale = self.D ** -0.5
        self.zero_rope = torch.zeros(self.D // 2, dtype=torch.float32, device=dev)  # Jamba attention has no RoPE
        get = _getter(weights)
        emb, fin, lay, bn, mix = _names(c)

        def g(n):
            return get(n).to(dev)

        def dv(t):
            return t.to(dev, bf).contiguous()

        def f32(t):
            return t.to(dev, torch.float32).contiguous()

        self.embed = dv(g(emb))
        self.norm = dv(g(fin))
        self.lm_head = self.embed if c.tie_word_embeddings else dv(g("lm_head.weight"))
        ones = lambda n: torch.ones(n, dtype=bf, device=dev)  # noqa: E731  (weightless RMSNorm)
        self.layers, n_attn, n_ssm = [], 0, 0
        for i in range(c.num_hidden_layers):
            p = lay.format(i=i)
            L = _Layer()
            L.ln1 = dv(g(p + bn + ".weight"))
            L.ln2 = L.w_gu = L.wd = L.moe = None
            L.attn = c.is_attention(i)
            if L.attn:
                a = p + "self_attn."
                L.idx, n_attn = n_attn, n_attn + 1
                L.wqkv = dv(torch.cat([g(a + "q_proj.weight"), g(a + "k_proj.weight"), g(a + "v_proj.weight")], 0))
                L.wo = dv(g(a + "o_proj.weight"))
            else:
                m = p + mix
                L.idx, n_ssm = n_ssm, n_ssm + 1
                L.w_in = dv(g(m + "in_proj.weight"))
                L.conv_w = f32(g(m + "conv1d.weight").reshape(c.inner, -1))
                L.conv_b = f32(g(m + "conv1d.bias")) if (m + "conv1d.bias") in weights else None
                L.w_x, L.w_dt = dv(g(m + "x_proj.weight")), dv(g(m + "dt_proj.weight"))
                L.dt_bias, L.A_log, L.Dp = f32(g(m + "dt_proj.bias")), f32(g(m + "A_log")), f32(g(m + "D"))
                L.wo = dv(g(m + "out_proj.weight"))
                L.n_dt = L.n_b = L.n_c = None
                if c.model_type == "jamba":
                    L.n_dt, L.n_b, L.n_c = (dv(g(m + n + "_layernorm.weight")) for n in ("dt", "b", "c"))
                elif c.model_type == "falcon_mamba":
                    L.n_dt, L.n_b, L.n_c = ones(c.time_step_rank), ones(c.state_size), ones(c.state_size)
            if c.model_type == "jamba":
                L.ln2 = dv(g(p + "pre_ff_layernorm.weight"))
                f = p + "feed_forward."
                if c.is_moe(i):
                    from .deepseek import expert_weights
                    src = _Prefixed(get, lambda n: n in weights, p[:-1] + ".feed_forward")
                    ws = [[t.to(dev).float() for t in expert_weights(src, "", e, c.intermediate_size)]
                          for e in range(c.num_experts)]
                    L.moe = (dv(g(f + "router.weight")), *pack_experts(*zip(*ws)))
                    del ws
                else:
                    L.w_gu = dv(ops.interleave_gate_up(g(f + "gate_proj.weight"), g(f + "up_proj.weight")))
                    L.wd = dv(g(f + "down_proj.weight"))
            self.layers.append(L)
        self.n_attn = n_attn

    def make_kv_cache(self, num_blocks: int, num_slots: int = 8) -> Mamba1Cache:
        return Mamba1Cache(self.cfg, num_blocks, num_slots, self.device)

    def kv_bytes_per_block(self) -> int:
        return 2 * max(1, self.n_attn) * self.hkv * BLOCK_SIZE * self.D * 2

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        from .. import ops
        return ops.linear(x, self.lm_head, out_dtype=torch.float32)

    def forward(self, fb, kv: Mamba1Cache) -> torch.Tensor:
        x = self.forward_hidden(fb, kv)
        if fb.logit_rows is not None:
            x = x.index_select(0, fb.logit_rows)
        return self.logits(x)

    def _attention(self, L, x, fb, kv):
        from .. import ops
        c = self.cfg
        T = x.shape[0]
        kc, vc = kv.layer(L.idx)
        q = ops.qkv_rope(ops.linear(x, L.wqkv), num_q_heads=c.num_attention_heads, num_kv_heads=c.num_key_value_heads,
                         head_dim=self.D, positions=fb.positions, inv_freq=self.zero_rope, slots=fb.slots,
                         k_cache=kc, v_cache=vc)
        o = torch.empty_like(q)
        nd = fb.num_decode
        if nd > 0:
            ops.decode_attention(q[:nd], kc, vc, fb.dec_block_tables, fb.dec_ctx_lens, scale=self.scale, out=o[:nd])
        if T > nd:
            ops.prefill_attention(q[nd:], kc, vc, fb.pre_block_tables, fb.pre_ctx_lens, fb.pre_cu_q, fb.pre_max_q,
                                  scale=self.scale, out=o[nd:])
        return o.view(T, -1)

    def _mixer(self, L, x, fb, kv, cu, slots):
        from .. import ops
        from ..ops._ext import ext
        c = self.cfg
        T, Di, N, R = x.shape[0], c.inner, c.state_size, c.time_step_rank
        xz = ops.linear(x, L.w_in)  # [T, x | z]
        xs = torch.empty(T, Di, dtype=torch.bfloat16, device=x.device)
        ext().mamba_conv(cu, slots, fb.positions, xz, L.conv_w, L.conv_b, kv.conv[L.idx], xs)
        p = ops.linear(xs, L.w_x)  # [T, dt | B | C]
        dt_r, bc = p[:, :R], p[:, R:]
        if L.n_dt is not None:  # Jamba / Falcon-Mamba: RMSNorm on dt, B and C
            eps = c.rms_norm_eps if c.model_type == "jamba" else c.mixer_rms_eps
            dt_r = ops.rmsnorm(dt_r.contiguous(), L.n_dt, eps)
            bc = torch.cat([ops.rmsnorm(p[:, R:R + N].contiguous(), L.n_b, eps),
                            ops.rmsnorm(p[:, R + N:].contiguous(), L.n_c, eps)], 1)
        dt = ops.linear(dt_r if dt_r.stride(0) % 8 == 0 else dt_r.contiguous(), L.w_dt)
        y = torch.empty(T, Di, dtype=torch.bfloat16, device=x.device)
        ext().mamba_scan(cu, slots, fb.positions, xs, dt, L.dt_bias, bc, N, L.A_log, L.Dp, xz[:, Di:],
                         kv.ssm[L.idx], y)
        ops._count(2)
        return y

    def _moe(self, L, x, h, nw):
        from .. import ops
        from .moe import routed_experts, softmax_topk
        c = self.cfg
        router, gu_w, gu_exp, dn_w, dn_exp = L.moe
        experts, weights = softmax_topk(ops.linear(x, router, out_dtype=torch.float32), c.num_experts_per_tok, False)
        out = routed_experts(x, experts, weights, gu_w, gu_exp, dn_w, dn_exp, c.num_experts, c.intermediate_size)
        return ops.rmsnorm(out, nw, c.rms_norm_eps, residual=h, residual_out=h)

    def forward_hidden(self, fb, kv: Mamba1Cache) -> torch.Tensor:
        from .. import ops
        from .decoder import LocalComm
        c = self.cfg
        comm = LocalComm(c.rms_norm_eps)
        nd = fb.num_decode
        dev = self.device
        if fb.pre_cu_q is None:  # decode only (also under CUDA-graph capture): one token per sequence
            cu = torch.arange(nd + 1, dtype=torch.int32, device=dev)
        elif nd:
            cu = torch.cat([torch.arange(nd, dtype=torch.int32, device=dev), fb.pre_cu_q + nd])
        else:
            cu = fb.pre_cu_q.contiguous()
        slots = fb.seq_slots
        if slots is None:
            slots = torch.arange(cu.numel() - 1, dtype=torch.int32, device=dev)
        slots = slots.long()
        h = ops.embedding(fb.input_ids, self.embed)
        x = ops.rmsnorm(h, self.layers[0].ln1, c.rms_norm_eps)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            a = self._attention(L, x, fb, kv) if L.attn else self._mixer(L, x, fb, kv, cu, slots)
            nw = self.layers[i + 1].ln1 if i + 1 < n else self.norm
            if L.ln2 is None:
                x = comm.rowpar_add_norm(a, L.wo, h, nw)
                continue
            x = comm.rowpar_add_norm(a, L.wo, h, L.ln2)
            if L.moe is not None:
                x = self._moe(L, x, h, nw)
                continue
            if x.shape[0] <= ops.ACC_MAX_M:
                gu = ops.swiglu_acc(ops.linear_acc(x, L.w_gu))
            else:
                gu = ops.linear_swiglu(x, L.w_gu)
            x = comm.rowpar_add_norm(gu, L.wd, h, nw)
        return x
