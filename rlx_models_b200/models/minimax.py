"""MiniMax-Text-01: lightning-attention / softmax-attention hybrid with a
Mixtral-style MoE in every layer (transformers ``minimax``).

    layer    x  = rmsnorm(h)                      (the residual is the NORMED input)
             h  = a_attn * x + b_attn * mixer(x)
             x2 = rmsnorm(h);  h = a_mlp * x2 + b_mlp * moe(x2)
    mixer    "full_attention": GQA with RoPE (optional sliding window)
             "linear_attention" (lightning attention, head width D):
                 [q | k | v] = silu(x W_qkv) per head
                 S_t = exp(-s) S_{t-1} + k_t^T v_t,   o_t = q_t S_t
                 out = W_out (rmsnorm(o) * sigmoid(x W_gate))   (norm over all heads)
             s = 2^(-8 (h+1) / H) * (1 - l / (L - 1) + 1e-5) for head h of layer l
    moe      softmax router, top-k, weights renormalised over the k; SwiGLU experts

Lightning attention is linear attention with a constant scalar decay per head,
i.e. the Mamba-2 SSD recurrence with dt = 1, A = -s, B = k, C = q, x = v and
D = 0. The GPU model therefore runs

  * prefill through the chunked form (``decay_attention_chunked``, the
    in-chunk decay matrix exp(G_i - G_j) and the carried state), and
  * decode through the SSD decode kernel (``ssd_decode_kernel``): the qkv
    GEMM's rows are reordered to the kernel's [x | B | C] = [v | k | q] row
    layout, followed by a block of zero rows whose outputs the kernel reads
    as dt_raw (dt_bias = log(e - 1) makes softplus(dt_raw + dt_bias) = 1),
    and the output-gate rows (one GEMM for all four products); the kernel's
    depthwise conv is given the identity taps [0, 1] so that its
    silu(conv(x)) is exactly the model's silu(x).

Per sequence the state slot holds that [H, D, D] fp32 state (the kernel's
[N, P] = [k dim, v dim] order) and the kernel's (unused) conv window.

Checkpoint names: transformers' MiniMaxForCausalLM (fused expert banks
``mlp.experts.gate_up_proj`` / ``down_proj``) or the release's
``block_sparse_moe.experts.{e}.w1 / w3 / w2``; the release's config keys
(``attn_type_list``, ``layernorm_*_alpha / beta``) are read as well.

Reference: crates/rlx-minimax (MiniMax lightning-attention runner: config +
per-layer lightning-attention step with a state side output, README
"rlx-minimax"); transformers' MiniMaxForCausalLM is the CPU oracle.
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
from .mamba2 import decay_attention_chunked

# softplus(DT_ONE) == 1: the SSD kernel's dt for a zero dt_raw column
DT_ONE = math.log(math.e - 1.0)
LIGHTNING_NORM_EPS = 1e-6  # the lightning output norm is built with the default eps, not rms_norm_eps


@dataclass
class MiniMaxConfig:
    model_type: str = "minimax"
    vocab_size: int = 200064
    hidden_size: int = 6144
    num_hidden_layers: int = 80
    num_attention_heads: int = 64
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 9216
    num_local_experts: int = 32
    num_experts_per_tok: int = 2
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000000.0
    rotary_dim: int = 0  # 0: the whole head (transformers' MiniMax rotary embedding)
    max_position_embeddings: int = 4096 * 32
    sliding_window: int | None = None
    block_size: int = 256
    layer_types: list = field(default_factory=list)
    full_attn_alpha_factor: float = 1.0
    full_attn_beta_factor: float = 1.0
    linear_attn_alpha_factor: float = 1.0
    linear_attn_beta_factor: float = 1.0
    mlp_alpha_factor: float = 1.0
    mlp_beta_factor: float = 1.0
    tie_word_embeddings: bool = False
    bos_token_id: int | None = 1
    eos_token_id: int | list | None = 2

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = ["full_attention" if (i + 1) % 2 else "linear_attention"
                                for i in range(self.num_hidden_layers)]

    def is_linear(self, i: int) -> bool:
        return self.layer_types[i] == "linear_attention"

    @property
    def attn_layer_indices(self) -> list:
        return [i for i in range(self.num_hidden_layers) if not self.is_linear(i)]

    def factors(self, i: int) -> tuple[float, float]:
        if self.is_linear(i):
            return float(self.linear_attn_alpha_factor), float(self.linear_attn_beta_factor)
        return float(self.full_attn_alpha_factor), float(self.full_attn_beta_factor)

    def slopes(self, i: int) -> torch.Tensor:
        """Per-head decay rate s of lightning layer i (fp32 [H])."""
        H = self.num_attention_heads
        base = 1.0 / (2 ** (8.0 / H))
        factor = 1 - i / (self.num_hidden_layers - 1 + 1e-5) + 1e-5
        return (base ** (torch.arange(H, dtype=torch.float64) + 1) * factor).float()

    @classmethod
    def from_dict(cls, d: dict) -> "MiniMaxConfig":
        d = dict(d)
        kw = {f.name: d[f.name] for f in fields(cls) if f.name in d and d[f.name] is not None}
        rp = d.get("rope_parameters") or {}
        if "rope_theta" in rp:
            kw["rope_theta"] = rp["rope_theta"]
        if not d.get("layer_types") and d.get("attn_type_list"):  # release config: 1 softmax, 0 lightning
            kw["layer_types"] = ["full_attention" if t else "linear_attention" for t in d["attn_type_list"]]
        for new, old in (("full_attn_alpha_factor", "layernorm_full_attention_alpha"),
                         ("full_attn_beta_factor", "layernorm_full_attention_beta"),
                         ("linear_attn_alpha_factor", "layernorm_linear_attention_alpha"),
                         ("linear_attn_beta_factor", "layernorm_linear_attention_beta"),
                         ("mlp_alpha_factor", "layernorm_mlp_alpha"),
                         ("mlp_beta_factor", "layernorm_mlp_beta")):
            if new not in d and old in d:
                kw[new] = d[old]
        if not kw.get("head_dim"):
            kw["head_dim"] = kw.get("hidden_size", cls.hidden_size) // kw.get("num_attention_heads",
                                                                               cls.num_attention_heads)
        if kw.get("num_key_value_heads") is None:
            kw["num_key_value_heads"] = kw.get("num_attention_heads", cls.num_attention_heads)
        return cls(**kw)

    @classmethod
    def from_file(cls, path: str) -> "MiniMaxConfig":
        with open(os.path.join(path, "config.json") if os.path.isdir(path) else path) as f:
            return cls.from_dict(json.load(f))


def is_minimax_config(path: str) -> bool:
    p = os.path.join(path, "config.json") if os.path.isdir(path) else path
    try:
        with open(p) as f:
            return json.load(f).get("model_type") in ("minimax", "minimax_text_01")
    except (OSError, ValueError):
        return False


def _getter(weights):
    return (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])


def _has(weights, n: str) -> bool:
    return n in weights


def expert_bank(get, has, m: str, e: int, I: int):
    """(gate [I, H], up [I, H], down [H, I]) of expert e of the MoE block at prefix m."""
    if has(m + "experts.gate_up_proj"):
        gu = get(m + "experts.gate_up_proj")[e]
        return gu[:I], gu[I:], get(m + "experts.down_proj")[e]
    b = m.replace("mlp.", "block_sparse_moe.") + f"experts.{e}."
    return get(b + "w1.weight"), get(b + "w3.weight"), get(b + "w2.weight")


def router_weight(get, has, m: str):
    return get(m + "gate.weight") if has(m + "gate.weight") else get(m.replace("mlp.", "block_sparse_moe.")
                                                                       + "gate.weight")


def random_weights(cfg: MiniMaxConfig, seed: int = 0, device="cpu", dtype=torch.bfloat16) -> dict:
    """transformers-named random weights (fused expert banks)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    H, D, nh, nkv = cfg.hidden_size, cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    E, I = cfg.num_local_experts, cfg.intermediate_size
    w = {}

    def t(name, *shape, std=0.02):
        w[name] = (torch.randn(*shape, generator=g) * std).to(device, dtype)

    def ones(name, n):
        w[name] = (1.0 + 0.1 * torch.randn(n, generator=g)).to(device, dtype)

    t("model.embed_tokens.weight", cfg.vocab_size, H)
    ones("model.norm.weight", H)
    if not cfg.tie_word_embeddings:
        t("lm_head.weight", cfg.vocab_size, H)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        ones(p + "input_layernorm.weight", H)
        ones(p + "post_attention_layernorm.weight", H)
        a = p + "self_attn."
        if cfg.is_linear(i):
            t(a + "qkv_proj.weight", 3 * nh * D, H)
            t(a + "output_gate.weight", nh * D, H)
            t(a + "out_proj.weight", H, nh * D)
            ones(a + "norm.weight", nh * D)
        else:
            t(a + "q_proj.weight", nh * D, H)
            t(a + "k_proj.weight", nkv * D, H)
            t(a + "v_proj.weight", nkv * D, H)
            t(a + "o_proj.weight", H, nh * D)
        t(p + "mlp.gate.weight", E, H)
        t(p + "mlp.experts.gate_up_proj", E, 2 * I, H)
        t(p + "mlp.experts.down_proj", E, H, I)
    return w


def _rope(x: torch.Tensor, pos: torch.Tensor, inv: torch.Tensor, mult: float) -> torch.Tensor:
    """Half-split RoPE on the first 2 * len(inv) dims of x [T, heads, D]."""
    r = 2 * inv.shape[0]
    f = pos.float()[:, None] * inv[None]
    cos, sin = (f.cos() * mult)[:, None], (f.sin() * mult)[:, None]
    x1, x2, rest = x[..., : r // 2], x[..., r // 2: r], x[..., r:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin, rest], -1)


class MiniMaxOracle:
    """fp32 forward over a chunk of tokens with carried state: lightning layers
    keep S [H, D, D], softmax layers their K / V rows. ``logits(ids)`` is the
    full-sequence forward; ``step(ids, state)`` continues from a state."""

    def __init__(self, cfg: MiniMaxConfig, weights, device="cpu"):
        self.cfg, self.device = cfg, torch.device(device)
        self.get, self.has = _getter(weights), (lambda n: _has(weights, n))
        self.inv, self.mult = rope_inv_freq(cfg.rotary_dim or cfg.head_dim, cfg.rope_theta, None,
                                            cfg.max_position_embeddings)
        self.inv = self.inv.to(self.device)

    def _t(self, n):
        return self.get(n).to(self.device, torch.float32)

    def _rms(self, x, w, eps):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    def _lightning(self, i, p, x, S):
        c = self.cfg
        T, nh, D = x.shape[0], c.num_attention_heads, c.head_dim
        qkv = F.silu(x @ self._t(p + "qkv_proj.weight").t()).view(T, nh, 3, D)
        q, k, v = (qkv[:, :, j].transpose(0, 1) for j in range(3))  # [H, T, D]
        g = (-c.slopes(i).to(self.device))[:, None].expand(nh, T)
        o, S = decay_attention_chunked(q, k, v, g, S, chunk=c.block_size)
        o = o.transpose(0, 1).reshape(T, nh * D)
        o = self._rms(o, self._t(p + "norm.weight"), LIGHTNING_NORM_EPS)
        o = torch.sigmoid(x @ self._t(p + "output_gate.weight").t()) * o
        return o @ self._t(p + "out_proj.weight").t(), S

    def _softmax_attn(self, p, x, pos, kv):
        c = self.cfg
        T, nh, nkv, D = x.shape[0], c.num_attention_heads, c.num_key_value_heads, c.head_dim
        q = _rope((x @ self._t(p + "q_proj.weight").t()).view(T, nh, D), pos, self.inv, self.mult)
        k = _rope((x @ self._t(p + "k_proj.weight").t()).view(T, nkv, D), pos, self.inv, self.mult)
        v = (x @ self._t(p + "v_proj.weight").t()).view(T, nkv, D)
        if kv is not None:
            k, v = torch.cat([kv[0], k]), torch.cat([kv[1], v])
        n = k.shape[0]
        qpos = pos[:, None]
        kpos = torch.arange(n, device=x.device)[None]
        mask = kpos <= qpos
        if c.sliding_window:
            mask &= kpos > qpos - c.sliding_window
        rep = nh // nkv
        kk, vv = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
        s = torch.einsum("thd,nhd->htn", q, kk) * D ** -0.5
        s = s.masked_fill(~mask[None], float("-inf")).softmax(-1)
        o = torch.einsum("htn,nhd->thd", s, vv).reshape(T, nh * D)
        return o @ self._t(p + "o_proj.weight").t(), (k, v)

    def _moe(self, p, x):
        c = self.cfg
        m = p + "mlp."
        probs = (x @ self._t_router(m).t()).softmax(-1)
        w, idx = probs.topk(c.num_experts_per_tok, -1)
        w = w / w.sum(-1, keepdim=True)
        out = torch.zeros_like(x)
        for e in idx.unique().tolist():
            rows, slot = (idx == e).nonzero(as_tuple=True)
            gt, up, dn = (t.to(self.device, torch.float32)
                          for t in expert_bank(self.get, self.has, m, e, c.intermediate_size))
            y = (F.silu(x[rows] @ gt.t()) * (x[rows] @ up.t())) @ dn.t()
            out.index_add_(0, rows, y * w[rows, slot, None])
        return out

    def _t_router(self, m):
        return router_weight(self.get, self.has, m).to(self.device, torch.float32)

    @torch.no_grad()
    def step(self, ids, state=None):
        """Logits [T, V] of tokens ``ids`` that follow ``state`` (None: a fresh
        sequence) and the state after them: {"pos": n, layer: S or (K, V)}."""
        c = self.cfg
        ids = torch.as_tensor(ids, device=self.device).long().view(-1)
        state = dict(state) if state is not None else {"pos": 0}
        start = state["pos"]
        pos = torch.arange(start, start + ids.shape[0], device=self.device)
        h = self._t("model.embed_tokens.weight")[ids]
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            x = self._rms(h, self._t(p + "input_layernorm.weight"), c.rms_norm_eps)
            if c.is_linear(i):
                a, state[i] = self._lightning(i, p + "self_attn.", x, state.get(i))
            else:
                a, state[i] = self._softmax_attn(p + "self_attn.", x, pos, state.get(i))
            al, be = c.factors(i)
            h = x * al + a * be
            x = self._rms(h, self._t(p + "post_attention_layernorm.weight"), c.rms_norm_eps)
            h = x * c.mlp_alpha_factor + self._moe(p, x) * c.mlp_beta_factor
        h = self._rms(h, self._t("model.norm.weight"), c.rms_norm_eps)
        head = self._t("model.embed_tokens.weight" if c.tie_word_embeddings else "lm_head.weight")
        state["pos"] = start + ids.shape[0]
        return h @ head.t(), state

    def logits(self, ids) -> torch.Tensor:
        return self.step(ids)[0]


def pack_lightning(cfg: MiniMaxConfig, w_qkv: torch.Tensor, w_gate: torch.Tensor) -> tuple[torch.Tensor, int]:
    """One input-projection matrix for a lightning layer in the SSD decode
    kernel's row order: [v (all heads) | k | q | Z zero rows | output gate],
    Z = H rounded up to 64 (the zero rows produce the kernel's dt_raw column).
    Returns (w [4 H D + Z, hidden], Z)."""
    nh, D = cfg.num_attention_heads, cfg.head_dim
    q, k, v = w_qkv.view(nh, 3, D, -1).unbind(1)
    Z = -(-nh // 64) * 64
    zero = w_qkv.new_zeros(Z, w_qkv.shape[1])
    return torch.cat([v.reshape(nh * D, -1), k.reshape(nh * D, -1), q.reshape(nh * D, -1), zero, w_gate], 0), Z


class MiniMaxCache:
    """Paged KV for the softmax-attention layers + per-slot lightning state."""

    def __init__(self, cfg: MiniMaxConfig, num_blocks: int, num_slots: int, device):
        n_attn = len(cfg.attn_layer_indices)
        n_lin = cfg.num_hidden_layers - n_attn
        nh, D = cfg.num_attention_heads, cfg.head_dim
        self.paged = PagedKVCache(max(1, n_attn), num_blocks if n_attn else 1, cfg.num_key_value_heads, D, device)
        self.k, self.v = self.paged.k, self.paged.v
        self.num_slots = num_slots
        # the SSD kernel's conv window (width 1: identity taps never read it into the result)
        self.conv = torch.zeros(max(1, n_lin), num_slots, 2, 3 * nh * D, 1, dtype=torch.bfloat16, device=device)
        self.ssm = torch.zeros(max(1, n_lin), num_slots, nh, D, D, dtype=torch.float32, device=device)

    def layer(self, i: int):
        return self.paged.layer(i)


class _Layer:
    __slots__ = ("ln1", "ln2", "idx", "linear", "wqkv", "wo", "w_in", "Z", "conv_w", "A_log", "dt_bias", "Dp",
                 "neg_slope", "norm_w", "alpha", "router", "gu_w", "gu_exp", "dn_w", "dn_exp")


class MiniMaxLM:
    """MiniMax-Text-01 on the package's kernels: tcgen05 GEMMs, the SSD decode
    kernel for lightning decode, paged attention for the softmax layers, the
    grouped MXFP4 expert GEMM for the MoE (softmax top-k routing kernel)."""
    stateful = True

    def __init__(self, cfg: MiniMaxConfig, weights, device="cuda"):
        from .. import ops
        from .moe import pack_experts
        self.cfg, self.device = cfg, torch.device(device)
        c, dev, bf = cfg, self.device, torch.bfloat16
        get, has = _getter(weights), (lambda n: _has(weights, n))
        inv, self.rope_mult = rope_inv_freq(c.rotary_dim or c.head_dim, c.rope_theta, None,
                                            c.max_position_embeddings)
        self.inv_freq = inv.to(dev)
        self.scale = c.head_dim ** -0.5
        self.nh, self.D, self.hkv = c.num_attention_heads, c.head_dim, c.num_key_value_heads
        dv = lambda t: t.to(dev, bf).contiguous()  # noqa: E731
        f32 = lambda t: t.to(dev, torch.float32).contiguous()  # noqa: E731
        self.embed = dv(get("model.embed_tokens.weight"))
        self.norm = dv(get("model.norm.weight"))
        self.lm_head = self.embed if c.tie_word_embeddings else dv(get("lm_head.weight"))
        self.layers, n_attn, n_lin = [], 0, 0
        for i in range(c.num_hidden_layers):
            p, L = f"model.layers.{i}.", _Layer()
            a = p + "self_attn."
            L.ln1, L.ln2 = dv(get(p + "input_layernorm.weight")), dv(get(p + "post_attention_layernorm.weight"))
            L.alpha, beta = c.factors(i)
            L.linear = c.is_linear(i)
            if L.linear:
                L.idx, n_lin = n_lin, n_lin + 1
                w_in, L.Z = pack_lightning(c, get(a + "qkv_proj.weight").float(), get(a + "output_gate.weight").float())
                L.w_in = dv(w_in)
                conv_dim = 3 * self.nh * self.D
                L.conv_w = torch.zeros(conv_dim, 2, dtype=torch.float32, device=dev)
                L.conv_w[:, 1] = 1.0
                s = c.slopes(i)
                L.A_log, L.neg_slope = f32(s.log()), f32(-s)
                L.dt_bias = torch.full((self.nh,), DT_ONE, dtype=torch.float32, device=dev)
                L.Dp = torch.zeros(self.nh, dtype=torch.float32, device=dev)
                L.norm_w = dv(get(a + "norm.weight"))
                L.wo = dv(get(a + "out_proj.weight").float() * beta)
            else:
                L.idx, n_attn = n_attn, n_attn + 1
                L.wqkv = dv(torch.cat([get(a + "q_proj.weight"), get(a + "k_proj.weight"),
                                       get(a + "v_proj.weight")], 0))
                L.wo = dv(get(a + "o_proj.weight").float() * beta)
            m = p + "mlp."
            L.router = f32(router_weight(get, has, m))
            banks = [expert_bank(get, has, m, e, c.intermediate_size) for e in range(c.num_local_experts)]
            L.gu_w, L.gu_exp, L.dn_w, L.dn_exp = (t.to(dev) for t in pack_experts(
                [b[0].float() for b in banks], [b[1].float() for b in banks], [b[2].float() for b in banks]))
            del banks
            self.layers.append(L)
        self.n_attn = n_attn
        self._ops = ops

    def make_kv_cache(self, num_blocks: int, num_slots: int = 8) -> MiniMaxCache:
        return MiniMaxCache(self.cfg, num_blocks, num_slots, self.device)

    def kv_bytes_per_block(self) -> int:
        return 2 * max(1, self.n_attn) * self.hkv * BLOCK_SIZE * self.D * 2

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        return self._ops.linear(x, self.lm_head, out_dtype=torch.float32)

    def forward(self, fb, kv: MiniMaxCache) -> torch.Tensor:
        x = self.forward_hidden(fb, kv)
        if fb.logit_rows is not None:
            x = x.index_select(0, fb.logit_rows)
        return self.logits(x)

    def _attention(self, L, x, fb, kv):
        ops, c = self._ops, self.cfg
        T = x.shape[0]
        kc, vc = kv.layer(L.idx)
        q = ops.qkv_rope(ops.linear(x, L.wqkv), num_q_heads=self.nh, num_kv_heads=self.hkv, head_dim=self.D,
                         positions=fb.positions, inv_freq=self.inv_freq, rope_scale=self.rope_mult, slots=fb.slots,
                         k_cache=kc, v_cache=vc, rot_dim=c.rotary_dim)
        o = torch.empty_like(q)
        nd, win = fb.num_decode, c.sliding_window or 0
        if nd > 0:
            ops.decode_attention(q[:nd], kc, vc, fb.dec_block_tables, fb.dec_ctx_lens, scale=self.scale, window=win,
                                 out=o[:nd])
        if T > nd:
            ops.prefill_attention(q[nd:], kc, vc, fb.pre_block_tables, fb.pre_ctx_lens, fb.pre_cu_q, fb.pre_max_q,
                                  scale=self.scale, window=win, out=o[nd:])
        return ops.linear(o.view(T, -1), L.wo)

    def _lightning(self, L, x, fb, kv, slots):
        from ..ops._ext import ext
        ops = self._ops
        T, nh, D = x.shape[0], self.nh, self.D
        HD = nh * D
        proj = ops.linear(x, L.w_in)  # [T, v | k | q | zeros | gate]
        y = torch.empty(T, HD, dtype=torch.bfloat16, device=x.device)
        nd = fb.num_decode
        if nd > 0:
            ext().ssd_decode(proj[:nd], 0, 3 * HD, L.conv_w, None, L.A_log, L.dt_bias, L.Dp, 0.0, 3.0e38,
                             kv.conv[L.idx], kv.ssm[L.idx], slots[:nd], fb.positions[:nd], y[:nd], nh)
            ops._count(1)
        if T > nd:
            cu, ctx, sl = fb.pre_cu_q.tolist(), fb.pre_ctx_lens.tolist(), slots[nd:].tolist()
            for s, n_ctx in enumerate(ctx):
                a, b = nd + cu[s], nd + cu[s + 1]
                n = b - a
                start, slot = n_ctx - n, sl[s]
                vkq = F.silu(proj[a:b, :3 * HD].float()).to(torch.bfloat16).float().view(n, 3, nh, D)
                v, k, q = (vkq[:, j].transpose(0, 1) for j in range(3))
                g = L.neg_slope[:, None].expand(nh, n)
                o, S = decay_attention_chunked(q, k, v, g, kv.ssm[L.idx, slot] if start > 0 else None,
                                               chunk=self.cfg.block_size)
                kv.ssm[L.idx, slot] = S
                y[a:b] = o.transpose(0, 1).reshape(n, HD).to(torch.bfloat16)
        yn = ops.rmsnorm(y, L.norm_w, LIGHTNING_NORM_EPS)
        gate = proj[:, 3 * HD + L.Z:]
        return ops.linear((yn.float() * torch.sigmoid(gate.float())).to(torch.bfloat16), L.wo)

    def _moe(self, L, x):
        from .moe import routed_experts, softmax_topk
        c = self.cfg
        idx, wts = softmax_topk(x.float() @ L.router.t(), c.num_experts_per_tok, True)
        return routed_experts(x.contiguous(), idx, (wts * c.mlp_beta_factor).contiguous(), L.gu_w, L.gu_exp,
                              L.dn_w, L.dn_exp, c.num_local_experts, c.intermediate_size)

    def forward_hidden(self, fb, kv: MiniMaxCache) -> torch.Tensor:
        ops, c = self._ops, self.cfg
        slots = fb.seq_slots
        if slots is None:
            nseq = fb.num_decode + (0 if fb.pre_ctx_lens is None else fb.pre_ctx_lens.shape[0])
            slots = torch.arange(nseq, dtype=torch.int32, device=self.device)
        h = ops.embedding(fb.input_ids, self.embed)
        x = ops.rmsnorm(h, self.layers[0].ln1, c.rms_norm_eps)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            a = self._lightning(L, x, fb, kv, slots) if L.linear else self._attention(L, x, fb, kv)
            h = x * L.alpha if L.alpha != 1.0 else x.clone()
            x = ops.rmsnorm(a, L.ln2, c.rms_norm_eps, residual=h, residual_out=h)   # h = a x + b mixer(x)
            h = x * c.mlp_alpha_factor if c.mlp_alpha_factor != 1.0 else x.clone()
            nw = self.layers[i + 1].ln1 if i + 1 < n else self.norm
            x = ops.rmsnorm(self._moe(L, x), nw, c.rms_norm_eps, residual=h, residual_out=h)
        return x
