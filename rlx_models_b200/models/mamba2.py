"""Mamba-2 (SSD) models: ``mamba2`` (attention-free) and ``bamba`` (Mamba-2
layers interleaved with GQA attention, SwiGLU feed-forward in every layer).

Mamba-2 mixer (H heads of width P, G groups of state size N):

    [z | xBC | dt] = in_proj(rmsnorm(h))
    x, B, C        = split(silu(conv1d(xBC) + bias))        (kernel 4, causal, depthwise)
    dt             = clamp(softplus(dt + dt_bias));  A = -exp(A_log)
    S_t            = exp(dt_t A) S_{t-1} + dt_t x_t B_t^T   (per head; B, C shared by the group)
    y_t            = S_t C_t + D x_t
    out            = out_proj(rmsnorm(y * silu(z)) * w)     (norm over the whole width)

The recurrence is linear attention with a scalar per-head decay
(q = C, k = B, v = dt x, log decay dt A), so prefill uses the chunked form

    O  = exp(G) * (Q S0) + lower(Q K^T * D) V,   S1 = exp(G_C) S0 + (K * exp(G_C - G))^T V

(G the in-chunk cumulative log decay, D_ij = exp(G_i - G_j) for j <= i), and
decode runs one sm_100a kernel per layer (``ssd_decode_kernel`` in
``csrc/linear_attn/gdn.cu``): conv step, gates, state update and y + D x; the
gated norm follows in torch.

B200 layout: paged KV for the attention layers only; per sequence a state
slot with the conv windows (double-buffered by position parity) and the fp32
SSM state [H, N, P].

Reference: SURVEY's hybrid SSM families (Nemotron-H, Jamba, Mamba; crates
rlx-ssm); transformers ``mamba2`` / ``bamba`` are the CPU oracles.
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

SSM_TYPES = ("mamba2", "bamba", "nemotron_h")


@dataclass
class SSMConfig:
    model_type: str = "mamba2"
    vocab_size: int = 50280
    hidden_size: int = 2560
    num_hidden_layers: int = 64
    # Mamba-2 mixer
    num_heads: int = 80
    head_dim: int = 64
    state_size: int = 128
    n_groups: int = 1
    conv_kernel: int = 4
    use_conv_bias: bool = True
    use_bias: bool = False
    time_step_limit: tuple = (0.0, float("inf"))
    rms_norm_eps: float = 1e-5
    tie_word_embeddings: bool = False
    # bamba: attention layers + SwiGLU feed-forward
    attn_layer_indices: list = field(default_factory=list)
    num_attention_heads: int = 0
    num_key_value_heads: int = 0
    attn_head_dim: int = 0
    intermediate_size: int = 0
    rope_theta: float = 10000.0
    partial_rotary_factor: float = 1.0
    max_position_embeddings: int = 262144
    bos_token_id: int | None = None
    eos_token_id: int | list | None = None
    # nemotron_h: one mixer per block ("mamba" | "attention" | "moe"), NoPE
    # attention, group-wise gated norm, squared-ReLU MoE (sigmoid group routing)
    layer_types: list = field(default_factory=list)
    norm_groups: int = 1
    n_routed_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    moe_shared_expert_intermediate_size: int = 0
    moe_latent_size: int | None = None
    n_group: int = 1
    topk_group: int = 1
    norm_topk_prob: bool = True
    routed_scaling_factor: float = 1.0
    extra: dict = field(default_factory=dict)

    @property
    def intermediate(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def conv_dim(self) -> int:
        return self.intermediate + 2 * self.n_groups * self.state_size

    @property
    def has_ffn(self) -> bool:
        return self.model_type == "bamba"

    def is_attention(self, i: int) -> bool:
        return i in self.attn_layer_indices

    def is_moe(self, i: int) -> bool:
        return bool(self.layer_types) and self.layer_types[i] == "moe"

    def is_mlp(self, i: int) -> bool:
        return bool(self.layer_types) and self.layer_types[i] == "mlp"

    def is_mamba(self, i: int) -> bool:
        return not (self.is_attention(i) or self.is_moe(i) or self.is_mlp(i))

    @property
    def rotary_dim(self) -> int:
        return int(self.attn_head_dim * self.partial_rotary_factor)

    @classmethod
    def from_dict(cls, d: dict) -> "SSMConfig":
        d = dict(d)
        mt = d.get("model_type", "mamba2")
        kw = {f.name: d[f.name] for f in fields(cls) if f.name in d and f.name != "extra"}
        if mt == "bamba":
            for src, dst in (("mamba_n_heads", "num_heads"), ("mamba_d_head", "head_dim"),
                             ("mamba_d_state", "state_size"), ("mamba_n_groups", "n_groups"),
                             ("mamba_d_conv", "conv_kernel"), ("mamba_conv_bias", "use_conv_bias"),
                             ("mamba_proj_bias", "use_bias")):
                if src in d:
                    kw[dst] = d[src]
            kw["attn_head_dim"] = d.get("head_dim") or d["hidden_size"] // d["num_attention_heads"]
            kw.pop("head_dim", None)
            kw["head_dim"] = d.get("mamba_d_head", 64)
            rp = d.get("rope_parameters") or {}
            kw["rope_theta"] = float(rp.get("rope_theta", d.get("rope_theta", 10000.0)))
            # transformers' Bamba rotary embedding spans the whole head whatever
            # partial_rotary_factor says; the oracle follows it
            kw["partial_rotary_factor"] = 1.0
            kw["rms_norm_eps"] = d.get("rms_norm_eps", 1e-5)
        elif mt == "nemotron_h":
            lt = d.get("layers_block_type") or d.get("layer_types")
            if not lt:
                code = {"M": "mamba", "*": "attention", "E": "moe", "-": "mlp"}
                lt = [code[ch] for ch in d.get("hybrid_override_pattern", "ME*E")]
            kw["layer_types"] = list(lt)
            kw["num_hidden_layers"] = len(lt)
            kw["attn_layer_indices"] = [i for i, t in enumerate(lt) if t == "attention"]
            for src, dst in (("mamba_num_heads", "num_heads"), ("mamba_head_dim", "head_dim"),
                             ("ssm_state_size", "state_size"), ("n_groups", "n_groups"), ("mamba_n_groups", "n_groups"),
                             ("conv_kernel", "conv_kernel"), ("use_conv_bias", "use_conv_bias"),
                             ("use_bias", "use_bias")):
                if src in d:
                    kw[dst] = d[src]
            kw["attn_head_dim"] = d.get("head_dim") or d["hidden_size"] // d["num_attention_heads"]
            kw["head_dim"] = d.get("mamba_head_dim", 64)
            kw["norm_groups"] = kw.get("n_groups", 8)
            kw["partial_rotary_factor"] = 0.0  # no positional encoding in the attention layers
            kw["rms_norm_eps"] = d.get("layer_norm_epsilon", 1e-5)
        else:
            kw["rms_norm_eps"] = d.get("layer_norm_epsilon", d.get("rms_norm_eps", 1e-5))
        if "time_step_limit" in d:
            kw["time_step_limit"] = tuple(float(v) for v in d["time_step_limit"])
        return cls(**kw)

    @classmethod
    def from_file(cls, path: str) -> "SSMConfig":
        with open(os.path.join(path, "config.json") if os.path.isdir(path) else path) as f:
            return cls.from_dict(json.load(f))


def is_ssm_config(path: str) -> bool:
    p = os.path.join(path, "config.json") if os.path.isdir(path) else path
    try:
        with open(p) as f:
            return json.load(f).get("model_type") in SSM_TYPES
    except (OSError, ValueError):
        return False


def _getter(weights):
    return (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])


def decay_attention_chunked(q, k, v, g, state=None, chunk: int = 64):
    """Linear attention with a scalar log decay per step (Mamba-2 SSD):
    q, k [H, L, dk], v [H, L, dv], g [H, L]; state [H, dk, dv]. Returns
    (o [H, L, dv], state) of S_t = exp(g_t) S_{t-1} + k_t v_t^T, o_t = S_t^T q_t."""
    H, L, dk = k.shape
    dv = v.shape[-1]
    dev = v.device
    S = torch.zeros(H, dk, dv, dtype=torch.float32, device=dev) if state is None else state.float()
    pad = (-L) % chunk
    q, k, v = (F.pad(t.float(), (0, 0, 0, pad)) for t in (q, k, v))
    g = F.pad(g.float(), (0, pad))
    N = (L + pad) // chunk
    q, k, v = (t.view(H, N, chunk, -1) for t in (q, k, v))
    G = g.view(H, N, chunk).cumsum(-1)
    lower = torch.ones(chunk, chunk, dtype=torch.bool, device=dev).tril()
    Dm = (G[..., :, None] - G[..., None, :]).masked_fill(~lower, float("-inf")).exp()
    QK = (q @ k.transpose(-1, -2)) * Dm
    out = torch.empty(H, N, chunk, dv, dtype=torch.float32, device=dev)
    for n in range(N):
        out[:, n] = G[:, n].exp()[..., None] * (q[:, n] @ S) + QK[:, n] @ v[:, n]
        gl = G[:, n, -1]
        S = gl.exp()[:, None, None] * S + (k[:, n] * (gl[:, None] - G[:, n]).exp()[..., None]).transpose(-1, -2) @ v[:, n]
    return out.view(H, N * chunk, dv)[:, :L], S


def conv_window(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, window: torch.Tensor | None):
    """silu(depthwise causal conv + bias) of x [C, L] with a window [C, K-1]; returns (y in x's dtype, window)."""
    K = w.shape[1]
    if window is None:
        window = x.new_zeros(x.shape[0], K - 1)
    full = torch.cat([window.to(x.dtype), x], 1)
    y = F.conv1d(full[None].float(), w.float()[:, None, :], None if b is None else b.float(), groups=x.shape[0])[0]
    return F.silu(y).to(x.dtype), full[:, -(K - 1):]


def ssd_mixer_seq(cfg: SSMConfig, proj: torch.Tensor, conv_w, conv_b, A_log, dt_bias, Dp,
                  conv_win=None, state=None, chunk: int = 64):
    """One sequence through the SSD core: proj [L, z | xBC | dt] -> (y [L, I]
    fp32 before the gated norm, z, new conv window, new state)."""
    c = cfg
    I, GN, H, P, N = c.intermediate, c.n_groups * c.state_size, c.num_heads, c.head_dim, c.state_size
    L = proj.shape[0]
    z = proj[:, :I]
    xbc, win = conv_window(proj[:, I:I + c.conv_dim].t(), conv_w, conv_b, conv_win)
    x, Bm, Cm = xbc.t().float().split([I, GN, GN], -1)
    dt = F.softplus(proj[:, I + c.conv_dim:I + c.conv_dim + H].float() + dt_bias.float())
    dt = dt.clamp(c.time_step_limit[0], c.time_step_limit[1])
    A = -A_log.float().exp()
    rep = H // c.n_groups
    q = Cm.view(L, c.n_groups, N).repeat_interleave(rep, 1).transpose(0, 1)
    k = Bm.view(L, c.n_groups, N).repeat_interleave(rep, 1).transpose(0, 1)
    xh = x.view(L, H, P)
    v = (xh * dt[..., None]).transpose(0, 1)
    o, S = decay_attention_chunked(q, k, v, (dt * A).t(), state, chunk)
    y = o.transpose(0, 1) + Dp.float()[None, :, None] * xh
    return y.reshape(L, I), z, win, S


def gated_norm(y: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float, groups: int = 1) -> torch.Tensor:
    """rmsnorm(y * silu(z)) * w over the last dim (fp32), in ``groups`` equal
    slices each with its own mean square (Nemotron-H) or over the whole width."""
    t = y.float() * F.silu(z.float())
    g = t.view(*t.shape[:-1], groups, -1)
    return (g * torch.rsqrt(g.pow(2).mean(-1, keepdim=True) + eps)).view_as(t) * w.float()


def _names(cfg: SSMConfig):
    """(embed, final norm, layer prefix, block-norm, mixer prefix) names of the family."""
    if cfg.model_type in ("mamba2", "nemotron_h"):
        return "backbone.embeddings.weight", "backbone.norm_f.weight", "backbone.layers.{i}.", "norm", "mixer."
    return "model.embed_tokens.weight", "model.final_layernorm.weight", "model.layers.{i}.", "input_layernorm", \
        "mamba."


def random_weights(cfg: SSMConfig, seed: int = 0, device="cpu", dtype=torch.bfloat16) -> dict:
    gen = torch.Generator(device=device).manual_seed(seed)
    Hd = cfg.hidden_size
    emb, fin, lay, bn, mix = _names(cfg)
    w = {}

    def lin(name, o, i):
        w[name] = (torch.randn(o, i, generator=gen, device=device) / math.sqrt(i)).to(dtype)

    def vec(name, n, base=1.0, s=0.1):
        w[name] = (base + s * torch.randn(n, generator=gen, device=device)).to(dtype)

    w[emb] = torch.randn(cfg.vocab_size, Hd, generator=gen, device=device).to(dtype)
    vec(fin, Hd)
    if not cfg.tie_word_embeddings:
        lin("lm_head.weight", cfg.vocab_size, Hd)
    for i in range(cfg.num_hidden_layers):
        p = lay.format(i=i)
        vec(p + bn + ".weight", Hd)
        if cfg.has_ffn:
            vec(p + "pre_ff_layernorm.weight", Hd)
            lin(p + "feed_forward.gate_proj.weight", cfg.intermediate_size, Hd)
            lin(p + "feed_forward.up_proj.weight", cfg.intermediate_size, Hd)
            lin(p + "feed_forward.down_proj.weight", Hd, cfg.intermediate_size)
        if cfg.is_attention(i):
            a, D = p + "self_attn.", cfg.attn_head_dim
            lin(a + "q_proj.weight", cfg.num_attention_heads * D, Hd)
            lin(a + "k_proj.weight", cfg.num_key_value_heads * D, Hd)
            lin(a + "v_proj.weight", cfg.num_key_value_heads * D, Hd)
            lin(a + "o_proj.weight", Hd, cfg.num_attention_heads * D)
            continue
        m = p + mix
        lin(m + "in_proj.weight", cfg.intermediate + cfg.conv_dim + cfg.num_heads, Hd)
        w[m + "conv1d.weight"] = (torch.randn(cfg.conv_dim, 1, cfg.conv_kernel, generator=gen, device=device)
                                  * 0.5).to(dtype)
        if cfg.use_conv_bias:
            vec(m + "conv1d.bias", cfg.conv_dim, base=0.0)
        w[m + "A_log"] = torch.arange(1, cfg.num_heads + 1, device=device).float().log().to(dtype)
        vec(m + "dt_bias", cfg.num_heads, base=-1.0, s=0.5)
        vec(m + "D", cfg.num_heads)
        vec(m + "norm.weight", cfg.intermediate)
        lin(m + "out_proj.weight", Hd, cfg.intermediate)
    return w


class SSMOracle:
    """fp32 full-sequence forward."""

    def __init__(self, cfg: SSMConfig, weights, device="cpu", chunk: int = 64):
        if cfg.model_type == "nemotron_h" and "backbone.embeddings.weight" not in weights and hasattr(weights, "items"):
            # transformers keeps Nemotron-H under ``model.``; the released checkpoints use ``backbone.``
            weights = {("backbone." + k[6:] if k.startswith("model.") else k): v for k, v in weights.items()}
        self.cfg, self.device, self.chunk, self.get = cfg, torch.device(device), chunk, _getter(weights)
        self.has = lambda n: n in weights  # noqa: E731
        if cfg.attn_layer_indices and cfg.rotary_dim:
            self.inv, self.mult = rope_inv_freq(cfg.rotary_dim, cfg.rope_theta, None, cfg.max_position_embeddings)

    def _t(self, n):
        return self.get(n).to(self.device, torch.float32)

    def _rms(self, x, n):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps) * self._t(n)

    def _expert(self, m: str, e: int, which: str) -> torch.Tensor:
        fused = m + f"experts.{which}"
        return self._t(fused)[e] if self.has(fused) else self._t(m + f"experts.{e}.{which}.weight")

    def _moe(self, m: str, x: torch.Tensor) -> torch.Tensor:
        """Nemotron-H MoE: sigmoid group-limited routing with the correction bias,
        squared-ReLU experts (up -> relu^2 -> down, no gate), optionally in a
        latent width (fc1 / fc2 latent projections around the routed experts),
        plus a squared-ReLU shared expert on the block input."""
        from types import SimpleNamespace
        from .deepseek import route
        c = self.cfg
        spec = SimpleNamespace(scoring_func="sigmoid", topk_method="noaux_tc", n_group=c.n_group,
                               topk_group=c.topk_group, num_experts_per_tok=c.num_experts_per_tok,
                               norm_topk_prob=c.norm_topk_prob, routed_scaling_factor=c.routed_scaling_factor)
        idx, wts = route(spec, x @ self._t(m + "gate.weight").t(), self._t(m + "gate.e_score_correction_bias"))
        xl = x @ self._t(m + "fc1_latent_proj.weight").t() if self.has(m + "fc1_latent_proj.weight") else x
        out = torch.zeros_like(xl)
        for e in idx.unique().tolist():
            rows, slot = (idx == e).nonzero(as_tuple=True)
            y = torch.relu(xl[rows] @ self._expert(m, e, "up_proj").t()).square() @ self._expert(m, e, "down_proj").t()
            out.index_add_(0, rows, y * wts[rows, slot, None])
        if self.has(m + "fc2_latent_proj.weight"):
            out = out @ self._t(m + "fc2_latent_proj.weight").t()
        s = m + "shared_experts."
        return out + torch.relu(x @ self._t(s + "up_proj.weight").t()).square() @ self._t(s + "down_proj.weight").t()

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
            x = self._rms(h, p + bn + ".weight")
            if c.is_moe(i):
                h = h + self._moe(p + mix, x)
            elif c.is_mlp(i):  # Nemotron-H squared-ReLU MLP block
                m = p + mix
                h = h + torch.relu(x @ self._t(m + "up_proj.weight").t()).square() @ self._t(m + "down_proj.weight").t()
            elif c.is_attention(i):
                a, D, nh, nkv = p + ("mixer." if c.model_type == "nemotron_h" else "self_attn."), c.attn_head_dim, c.num_attention_heads, c.num_key_value_heads
                q = (x @ self._t(a + "q_proj.weight").t()).view(S, nh, D)
                k = (x @ self._t(a + "k_proj.weight").t()).view(S, nkv, D)
                if c.rotary_dim:
                    q, k = R.rope(q, pos, self.inv, self.mult), R.rope(k, pos, self.inv, self.mult)
                v = (x @ self._t(a + "v_proj.weight").t()).view(S, nkv, D)
                o = R.attention(q, k, v, pos, pos, D ** -0.5, causal=True).reshape(S, nh * D)
                h = h + o @ self._t(a + "o_proj.weight").t()
            else:
                m = p + mix
                proj = x @ self._t(m + "in_proj.weight").t()
                cb = self._t(m + "conv1d.bias") if self.has(m + "conv1d.bias") else None
                y, z, _, _ = ssd_mixer_seq(c, proj, self._t(m + "conv1d.weight")[:, 0], cb, self._t(m + "A_log"),
                                           self._t(m + "dt_bias"), self._t(m + "D"), chunk=self.chunk)
                h = h + gated_norm(y, z, self._t(m + "norm.weight"), c.rms_norm_eps, c.norm_groups) @ \
                    self._t(m + "out_proj.weight").t()
            if c.has_ffn:
                x = self._rms(h, p + "pre_ff_layernorm.weight")
                f = p + "feed_forward."
                h = h + (F.silu(x @ self._t(f + "gate_proj.weight").t()) * (x @ self._t(f + "up_proj.weight").t())) \
                    @ self._t(f + "down_proj.weight").t()
        h = self._rms(h, fin)
        head = emb if c.tie_word_embeddings else "lm_head.weight"
        return h @ self._t(head).t()


# ---------------------------------------------------------------------------
# GPU model (engine interface)
# ---------------------------------------------------------------------------

class SSMCache:
    """Paged KV for attention layers + per-slot conv windows and SSM states."""

    def __init__(self, cfg: SSMConfig, num_blocks: int, num_slots: int, device):
        n_attn = len(cfg.attn_layer_indices)
        n_ssm = sum(cfg.is_mamba(i) for i in range(cfg.num_hidden_layers))
        hkv, D = (cfg.num_key_value_heads, cfg.attn_head_dim) if n_attn else (1, 64)
        self.paged = PagedKVCache(max(1, n_attn), num_blocks if n_attn else 1, hkv, D, device)
        self.k, self.v = self.paged.k, self.paged.v
        self.num_slots = num_slots
        self.conv = torch.zeros(n_ssm, num_slots, 2, cfg.conv_dim, cfg.conv_kernel - 1, dtype=torch.bfloat16,
                                device=device)
        self.ssm = torch.zeros(n_ssm, num_slots, cfg.num_heads, cfg.state_size, cfg.head_dim, dtype=torch.float32,
                               device=device)

    def layer(self, i: int):
        return self.paged.layer(i)


class _BackboneNames:
    """A weight source with ``model.*`` names seen under ``backbone.*``."""

    def __init__(self, weights):
        self.w = weights
        self.map = {("backbone." + k[6:] if k.startswith("model.") else k): k for k in weights.keys()}

    def keys(self):
        return list(self.map)

    def __contains__(self, name):
        return name in self.map

    def take(self, name, **kw):
        n = self.map[name]
        return self.w.take(n, **kw) if hasattr(self.w, "take") else self.w[n]

    def __getitem__(self, name):
        return self.take(name)


class _Layer:
    __slots__ = ("ln1", "ln2", "w_gu", "wd", "wo", "attn", "idx", "wqkv", "w_in", "conv_w", "conv_b", "A_log",
                 "dt_bias", "Dp", "norm_w", "kind", "up", "moe")


class SSMHybridLM:
    stateful = True

    def __init__(self, cfg: SSMConfig, weights, device="cuda"):
        from .. import ops
        self.cfg, self.device = cfg, torch.device(device)
        c, dev, bf = cfg, self.device, torch.bfloat16
        self.hkv = c.num_key_value_heads or 1
        self.D = c.attn_head_dim or 64
        if c.attn_layer_indices:
            if c.rotary_dim:
                inv, self.rope_mult = rope_inv_freq(c.rotary_dim, c.rope_theta, None, c.max_position_embeddings)
            else:  # NoPE attention (Nemotron-H): zero frequencies rotate nothing
                inv, self.rope_mult = torch.zeros(c.attn_head_dim // 2), 1.0
            self.inv_freq = inv.to(dev)
            self.scale = c.attn_head_dim ** -0.5
        if c.model_type == "nemotron_h" and "backbone.embeddings.weight" not in weights:
            weights = _BackboneNames(weights)  # transformers' ``model.`` names -> the releases' ``backbone.``
        get = _getter(weights)
        self._weights = weights
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
        self.layers, n_attn, n_ssm = [], 0, 0
        for i in range(c.num_hidden_layers):
            p = lay.format(i=i)
            L = _Layer()
            L.ln1 = dv(g(p + bn + ".weight"))
            L.ln2 = L.w_gu = L.wd = None
            if c.has_ffn:
                L.ln2 = dv(g(p + "pre_ff_layernorm.weight"))
                f = p + "feed_forward."
                L.w_gu = dv(ops.interleave_gate_up(g(f + "gate_proj.weight"), g(f + "up_proj.weight")))
                L.wd = dv(g(f + "down_proj.weight"))
            L.attn = c.is_attention(i)
            L.kind = "attention" if L.attn else ("moe" if c.is_moe(i) else ("mlp" if c.is_mlp(i) else "mamba"))
            L.moe = None
            if L.kind == "mlp":  # Nemotron-H squared-ReLU MLP: h += relu(x W_up)^2 W_down
                L.up, L.wo = dv(g(p + mix + "up_proj.weight")), dv(g(p + mix + "down_proj.weight"))
            elif L.kind == "moe":
                L.moe = self._load_moe(g, dv, p + mix)
            elif L.attn:
                a = p + ("mixer." if c.model_type == "nemotron_h" else "self_attn.")
                L.idx, n_attn = n_attn, n_attn + 1
                L.wqkv = dv(torch.cat([g(a + "q_proj.weight"), g(a + "k_proj.weight"), g(a + "v_proj.weight")], 0))
                L.wo = dv(g(a + "o_proj.weight"))
            else:
                m = p + mix
                L.idx, n_ssm = n_ssm, n_ssm + 1
                L.w_in = dv(g(m + "in_proj.weight"))
                L.conv_w = f32(g(m + "conv1d.weight").reshape(c.conv_dim, -1))
                L.conv_b = f32(g(m + "conv1d.bias")) if (m + "conv1d.bias") in weights else None
                L.A_log, L.dt_bias, L.Dp = f32(g(m + "A_log")), f32(g(m + "dt_bias")), f32(g(m + "D"))
                L.norm_w = f32(g(m + "norm.weight"))
                L.wo = dv(g(m + "out_proj.weight"))
            self.layers.append(L)
        self.n_attn = n_attn

    def _load_moe(self, g, dv, m: str):
        """Nemotron-H MoE block: router + correction bias, squared-ReLU experts packed
        for the grouped MXFP4 GEMM with the gate rows set to the up rows (its epilogue
        computes u * g * sigmoid(alpha g); with g = u and a huge alpha that is
        relu(u) * u = relu(u)^2), latent projections, squared-ReLU shared expert."""
        from types import SimpleNamespace
        from .moe import pack_experts
        c = self.cfg
        dev = self.device
        E = c.n_routed_experts

        def bank(which):  # per-expert matrices from a fused [E, out, in] bank or per-expert tensors
            fused = m + f"experts.{which}"
            if fused in self._weights:
                b = g(fused).float()
                return [b[e] for e in range(E)]
            return [g(m + f"experts.{e}.{which}.weight").float() for e in range(E)]
        ups, downs = bank("up_proj"), bank("down_proj")
        gu_w, gu_exp, dn_w, dn_exp = pack_experts(ups, ups, downs)
        del ups, downs
        s = m + "shared_experts."
        return SimpleNamespace(
            router=g(m + "gate.weight").to(dev, torch.float32).contiguous(),
            corr=g(m + "gate.e_score_correction_bias").to(dev, torch.float32),
            gu_w=gu_w, gu_exp=gu_exp, dn_w=dn_w, dn_exp=dn_exp,
            fc1=dv(g(m + "fc1_latent_proj.weight")) if (m + "fc1_latent_proj.weight") in self._weights else None,
            fc2=dv(g(m + "fc2_latent_proj.weight")) if (m + "fc2_latent_proj.weight") in self._weights else None,
            sh_up=dv(g(s + "up_proj.weight")), sh_down=dv(g(s + "down_proj.weight")),
            spec=SimpleNamespace(scoring_func="sigmoid", topk_method="noaux_tc", n_group=c.n_group,
                                 topk_group=c.topk_group, num_experts_per_tok=c.num_experts_per_tok,
                                 norm_topk_prob=c.norm_topk_prob, routed_scaling_factor=c.routed_scaling_factor))

    def _moe(self, M, x: torch.Tensor) -> torch.Tensor:
        from .. import ops
        from .deepseek import route
        from .moe import routed_experts
        idx, wts = route(M.spec, x.float() @ M.router.t(), M.corr)
        xl = ops.linear(x, M.fc1) if M.fc1 is not None else x
        out = routed_experts(xl.contiguous(), idx.to(torch.int32).contiguous(), wts.float().contiguous(), M.gu_w,
                             M.gu_exp, M.dn_w, M.dn_exp, self.cfg.n_routed_experts,
                             self.cfg.moe_intermediate_size, alpha=1e30)
        if M.fc2 is not None:
            out = ops.linear(out, M.fc2)
        sh = torch.relu(ops.linear(x, M.sh_up).float()).square().to(x.dtype)
        return out + ops.linear(sh, M.sh_down)

    def make_kv_cache(self, num_blocks: int, num_slots: int = 8) -> SSMCache:
        return SSMCache(self.cfg, num_blocks, num_slots, self.device)

    def kv_bytes_per_block(self) -> int:
        return 2 * max(1, self.n_attn) * self.hkv * BLOCK_SIZE * self.D * 2

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        from .. import ops
        return ops.linear(x, self.lm_head, out_dtype=torch.float32)

    def forward(self, fb, kv: SSMCache) -> torch.Tensor:
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
                         head_dim=c.attn_head_dim, positions=fb.positions, inv_freq=self.inv_freq,
                         rope_scale=self.rope_mult, slots=fb.slots, k_cache=kc, v_cache=vc, rot_dim=c.rotary_dim)
        o = torch.empty_like(q)
        nd = fb.num_decode
        if nd > 0:
            ops.decode_attention(q[:nd], kc, vc, fb.dec_block_tables, fb.dec_ctx_lens, scale=self.scale, out=o[:nd])
        if T > nd:
            ops.prefill_attention(q[nd:], kc, vc, fb.pre_block_tables, fb.pre_ctx_lens, fb.pre_cu_q, fb.pre_max_q,
                                  scale=self.scale, out=o[nd:])
        return o.view(T, -1)

    def _ssm(self, L, x, fb, kv, slots):
        from .. import ops
        from ..ops._ext import ext
        c = self.cfg
        T = x.shape[0]
        I = c.intermediate
        proj = ops.linear(x, L.w_in)  # [T, z | xBC | dt]
        y = torch.empty(T, I, dtype=torch.bfloat16, device=x.device)
        nd = fb.num_decode
        if nd > 0:
            ext().ssd_decode(proj[:nd], I, I + c.conv_dim, L.conv_w, L.conv_b, L.A_log, L.dt_bias, L.Dp,
                             float(c.time_step_limit[0]), float(min(c.time_step_limit[1], 3.0e38)), kv.conv[L.idx],
                             kv.ssm[L.idx], slots[:nd], fb.positions[:nd], y[:nd], c.n_groups)
            ops._count(1)
        if T > nd:
            cu, ctx, sl = fb.pre_cu_q.tolist(), fb.pre_ctx_lens.tolist(), slots[nd:].tolist()
            for s, n_ctx in enumerate(ctx):
                a, b = nd + cu[s], nd + cu[s + 1]
                n = b - a
                start, slot = n_ctx - n, sl[s]
                win = kv.conv[L.idx, slot, start & 1] if start > 0 else None
                state = kv.ssm[L.idx, slot] if start > 0 else None  # [H, N, P], the kernel's layout
                yy, _, new_win, S = ssd_mixer_seq(c, proj[a:b], L.conv_w, L.conv_b, L.A_log, L.dt_bias, L.Dp, win,
                                                  state)
                kv.conv[L.idx, slot, (start + n) & 1] = new_win
                kv.ssm[L.idx, slot] = S
                y[a:b] = yy.to(torch.bfloat16)
        return gated_norm(y, proj[:, :I], L.norm_w, c.rms_norm_eps, c.norm_groups).to(torch.bfloat16)

    def forward_hidden(self, fb, kv: SSMCache) -> torch.Tensor:
        from .. import ops
        from .decoder import LocalComm
        c = self.cfg
        comm = LocalComm(c.rms_norm_eps)
        slots = fb.seq_slots
        if slots is None:
            nseq = fb.num_decode + (0 if fb.pre_ctx_lens is None else fb.pre_ctx_lens.shape[0])
            slots = torch.arange(nseq, dtype=torch.int32, device=self.device)
        h = ops.embedding(fb.input_ids, self.embed)
        x = ops.rmsnorm(h, self.layers[0].ln1, c.rms_norm_eps)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            nw = self.layers[i + 1].ln1 if i + 1 < n else self.norm
            if L.kind == "moe":  # h += moe(x); x = rmsnorm(h) for the next block
                x = ops.rmsnorm(self._moe(L.moe, x), nw, c.rms_norm_eps, residual=h, residual_out=h)
                continue
            if L.kind == "mlp":
                a = torch.relu(ops.linear(x, L.up).float()).square().to(x.dtype)
            else:
                a = self._attention(L, x, fb, kv) if L.attn else self._ssm(L, x, fb, kv, slots)
            if L.w_gu is None:
                x = comm.rowpar_add_norm(a, L.wo, h, nw)
                continue
            x = comm.rowpar_add_norm(a, L.wo, h, L.ln2)
            if x.shape[0] <= ops.ACC_MAX_M:
                gu = ops.swiglu_acc(ops.linear_acc(x, L.w_gu))
            else:
                gu = ops.linear_swiglu(x, L.w_gu)
            x = comm.rowpar_add_norm(gu, L.wd, h, nw)
        return x
