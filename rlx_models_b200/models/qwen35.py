"""Qwen3.5 hybrid decoder (``qwen3_5_text``): Gated DeltaNet linear-attention
layers interleaved with gated full-attention layers (every
``full_attention_interval``-th layer, 4 by default).

Gated DeltaNet layer (per value head h, key head h // (Hv / Hk)):

    [q | k | v] = silu(causal_conv1d(in_proj_qkv(x)))      (kernel 4, per channel)
    q, k        = l2norm(q), l2norm(k);  q *= dk^-1/2
    g_t         = -exp(A_log) * softplus(in_proj_a(x) + dt_bias)   (log decay)
    beta_t      = sigmoid(in_proj_b(x))
    S_t         = exp(g_t) S_{t-1} + k_t u_t^T,
    u_t         = beta_t (v_t - exp(g_t) S_{t-1}^T k_t)           (delta rule)
    o_t         = S_t^T q_t
    y           = out_proj(rmsnorm(o) * w * silu(in_proj_z(x)))

Full-attention layers: q_proj emits [query | gate] per head; QK RMSNorm with
(1 + w) weights; RoPE on the first quarter of each 256-wide head; the
attention output is multiplied by sigmoid(gate) before o_proj. All RMSNorms
except the gated one use (1 + w) weights. For text the three mRoPE position
axes coincide, so the rotary embedding is the ordinary one.

Prefill uses the chunked form of the recurrence (per chunk of C tokens, with
G the in-chunk cumulative log decay and D_ij = exp(G_i - G_j) for j <= i):

    A  = strictly-lower (K K^T * D)
    (I + diag(beta) A) [W_v | W_k] = [beta * V | beta * exp(G) * K]
    U  = W_v - W_k S0                      (the written values u_t)
    O  = exp(G) * (Q S0) + lower(Q K^T * D) U
    S1 = exp(G_C) S0 + (K * exp(G_C - G))^T U

which is the sequential recurrence regrouped (the unit-lower-triangular
system is solved with ``torch.linalg.solve_triangular``). Decode runs one
fused sm_100a kernel per layer (``csrc/linear_attn/gdn.cu``): conv1d step,
l2norm, gates, the delta-rule state update and the gated RMSNorm.

B200 layout: the paged KV cache holds only the full-attention layers; each
sequence owns a state slot with its conv window (double-buffered by position
parity so that value heads sharing a key head never race) and its fp32
recurrent state [Hv, dk, dv]. Prefix caching is off for this family (the
recurrent state is not per block).

Reference: crates/rlx-qwen35 (Gated DeltaNet + periodic attention + MTP:
the largest family of the reference); transformers ``qwen3_5`` is the
numerics oracle on CPU.
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

QWEN35_TYPES = ("qwen3_5_text", "qwen3_5", "qwen3_5_moe_text", "qwen3_5_moe", "qwen3_next")


@dataclass
class Qwen35Config:
    model_type: str = "qwen3_5_text"
    vocab_size: int = 248320
    hidden_size: int = 4096
    intermediate_size: int = 12288
    num_hidden_layers: int = 32
    num_attention_heads: int = 16
    num_key_value_heads: int = 4
    head_dim: int = 256
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e7
    partial_rotary_factor: float = 0.25
    max_position_embeddings: int = 32768
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    linear_conv_kernel_dim: int = 4
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 32
    layer_types: list | None = None
    # Qwen3.5-MoE (qwen3_5_moe_text): every MLP routed (softmax, top-k, renormalised)
    # plus a sigmoid-gated shared expert
    num_experts: int = 0
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 512
    shared_expert_intermediate_size: int = 512
    norm_topk_prob: bool = True
    mlp_only_layers: list = field(default_factory=list)  # Qwen3-Next: dense layers of a MoE model
    decoder_sparse_step: int = 1
    bos_token_id: int | None = None
    eos_token_id: int | list | None = None
    extra: dict = field(default_factory=dict)

    def __post_init__(self):
        if self.layer_types is None:
            self.layer_types = ["full_attention" if (i + 1) % 4 == 0 else "linear_attention"
                                for i in range(self.num_hidden_layers)]

    @property
    def key_dim(self) -> int:
        return self.linear_key_head_dim * self.linear_num_key_heads

    @property
    def value_dim(self) -> int:
        return self.linear_value_head_dim * self.linear_num_value_heads

    @property
    def conv_dim(self) -> int:
        return 2 * self.key_dim + self.value_dim

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def is_linear(self, i: int) -> bool:
        return self.layer_types[i] == "linear_attention"

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def is_moe_layer(self, i: int) -> bool:
        return self.is_moe and i not in self.mlp_only_layers and (i + 1) % self.decoder_sparse_step == 0

    @classmethod
    def from_dict(cls, d: dict) -> "Qwen35Config":
        d = dict(d)
        if isinstance(d.get("text_config"), dict):  # the multimodal wrapper: the text model's config
            moe = "moe" in str(d.get("model_type", ""))
            d = dict(d["text_config"], model_type=d["text_config"].get(
                "model_type", "qwen3_5_moe_text" if moe else "qwen3_5_text"))
        kw = {f.name: d[f.name] for f in fields(cls) if f.name in d and f.name != "extra"}
        rp = d.get("rope_parameters") or d.get("rope_scaling") or {}
        if "rope_theta" in rp:
            kw["rope_theta"] = float(rp["rope_theta"])
        if "partial_rotary_factor" in rp:
            kw["partial_rotary_factor"] = float(rp["partial_rotary_factor"])
        if kw.get("layer_types") is None:
            n, every = d["num_hidden_layers"], int(d.get("full_attention_interval", 4))
            kw["layer_types"] = ["full_attention" if (i + 1) % every == 0 else "linear_attention" for i in range(n)]
        return cls(**kw)

    @classmethod
    def from_file(cls, path: str) -> "Qwen35Config":
        with open(os.path.join(path, "config.json") if os.path.isdir(path) else path) as f:
            return cls.from_dict(json.load(f))

    def to_hf_dict(self) -> dict:
        d = {f.name: getattr(self, f.name) for f in fields(self) if f.name != "extra"}
        d["rope_parameters"] = {"rope_type": "default", "rope_theta": self.rope_theta,
                                "partial_rotary_factor": self.partial_rotary_factor}
        return d


def is_qwen35_config(path: str) -> bool:
    p = os.path.join(path, "config.json") if os.path.isdir(path) else path
    try:
        with open(p) as f:
            d = json.load(f)
    except (OSError, ValueError):
        return False
    return d.get("model_type") in QWEN35_TYPES


# ---------------------------------------------------------------------------
# shared math
# ---------------------------------------------------------------------------

def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gdn_gates(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    """(log decay g, write strength beta), both fp32 [..., Hv]."""
    g = -A_log.float().exp() * F.softplus(a.float() + dt_bias.float())
    return g, b.float().sigmoid()


def causal_conv1d(x: torch.Tensor, w: torch.Tensor, window: torch.Tensor | None = None):
    """x [C, L] (one sequence), w [C, K], window [C, K-1] (the inputs before x,
    oldest first; None = zeros). Returns (silu(conv) [C, L], new window)."""
    K = w.shape[1]
    if window is None:
        window = x.new_zeros(x.shape[0], K - 1)
    full = torch.cat([window.to(x.dtype), x], 1)
    y = F.conv1d(full[None].float(), w.float()[:, None, :], groups=x.shape[0])[0]
    return F.silu(y).to(x.dtype), full[:, -(K - 1):]


def gated_delta_recurrent(q, k, v, g, beta, state=None):
    """Token-by-token gated delta rule. q, k [H, L, dk] (normalised, q scaled),
    v [H, L, dv], g / beta [H, L]; state [H, dk, dv]. Returns (o [H, L, dv], state)."""
    H, L, dk = k.shape
    S = torch.zeros(H, dk, v.shape[-1], dtype=torch.float32, device=v.device) if state is None else state.float()
    out = []
    for t in range(L):
        S = S * g[:, t].exp()[:, None, None]
        u = beta[:, t, None] * (v[:, t].float() - torch.einsum("hkv,hk->hv", S, k[:, t].float()))
        S = S + k[:, t].float()[:, :, None] * u[:, None, :]
        out.append(torch.einsum("hkv,hk->hv", S, q[:, t].float()))
    return torch.stack(out, 1), S


def gated_delta_chunked(q, k, v, g, beta, state=None, chunk: int = 64):
    """Chunked gated delta rule (same contract as ``gated_delta_recurrent``)."""
    H, L, dk = k.shape
    dv = v.shape[-1]
    dev = v.device
    S = torch.zeros(H, dk, dv, dtype=torch.float32, device=dev) if state is None else state.float()
    pad = (-L) % chunk
    q, k, v = (F.pad(t.float(), (0, 0, 0, pad)) for t in (q, k, v))
    g, beta = F.pad(g.float(), (0, pad)), F.pad(beta.float(), (0, pad))
    N = (L + pad) // chunk
    q, k, v = (t.view(H, N, chunk, -1) for t in (q, k, v))
    g, beta = g.view(H, N, chunk), beta.view(H, N, chunk)
    G = g.cumsum(-1)
    lower = torch.ones(chunk, chunk, dtype=torch.bool, device=dev).tril()
    D = (G[..., :, None] - G[..., None, :]).masked_fill(~lower, float("-inf")).exp()  # [H, N, C, C]
    eye = torch.eye(chunk, device=dev)
    A = (k @ k.transpose(-1, -2)) * D * (1 - eye)
    M = eye + beta[..., :, None] * A
    rhs = torch.cat([beta[..., None] * v, (beta * G.exp())[..., None] * k], -1)
    W = torch.linalg.solve_triangular(M, rhs, upper=False, unitriangular=True)
    Wv, Wk = W[..., :dv], W[..., dv:]
    QK = (q @ k.transpose(-1, -2)) * D
    out = torch.empty(H, N, chunk, dv, dtype=torch.float32, device=dev)
    for n in range(N):
        U = Wv[:, n] - Wk[:, n] @ S
        out[:, n] = G[:, n].exp()[..., None] * (q[:, n] @ S) + QK[:, n] @ U
        gl = G[:, n, -1]
        S = gl.exp()[:, None, None] * S + (k[:, n] * (gl[:, None] - G[:, n]).exp()[..., None]).transpose(-1, -2) @ U
    return out.view(H, N * chunk, dv)[:, :L], S


def gated_rmsnorm(o: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """rmsnorm over the last dim (plain weight) times silu(z); fp32."""
    of = o.float()
    return of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + eps) * w.float() * F.silu(z.float())


def _getter(weights):
    return (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])


class CanonicalSource:
    """Checkpoint tensors under the names the builders read.

    * released multimodal checkpoints keep the text model under
      ``model.language_model.``: mapped to ``model.``; the vision tower and the
      MTP head are dropped;
    * Qwen3-Next fuses the Gated DeltaNet input projections per key-head group
      (``in_proj_qkvz`` rows [q | k | v of the group's value heads | z of
      them] per group, ``in_proj_ba`` rows [b | a] per group): regrouped into
      Qwen3.5's ``in_proj_qkv`` ([all q | all k | all v]), ``in_proj_z``,
      ``in_proj_b`` and ``in_proj_a``."""

    def __init__(self, weights, cfg: Qwen35Config):
        self.get, self.cfg = _getter(weights), cfg
        self.map: dict[str, tuple] = {}
        for n in list(weights.keys()):
            if n.startswith(("model.visual.", "mtp.")):
                continue
            c = n.replace("model.language_model.", "model.", 1)
            if c.endswith("linear_attn.in_proj_qkvz.weight"):
                pre = c[: -len("in_proj_qkvz.weight")]
                for part in ("in_proj_qkv", "in_proj_z"):
                    self.map[pre + part + ".weight"] = (n, part)
            elif c.endswith("linear_attn.in_proj_ba.weight"):
                pre = c[: -len("in_proj_ba.weight")]
                for part in ("in_proj_b", "in_proj_a"):
                    self.map[pre + part + ".weight"] = (n, part)
            else:
                self.map[c] = (n, None)

    def keys(self):
        return list(self.map)

    def __contains__(self, name):
        return name in self.map

    def __getitem__(self, name):
        n, part = self.map[name]
        t = self.get(n)
        if part is None:
            return t
        c = self.cfg
        Hk, dk, dv = c.linear_num_key_heads, c.linear_key_head_dim, c.linear_value_head_dim
        r = c.linear_num_value_heads // Hk
        H = t.shape[-1]
        if part in ("in_proj_qkv", "in_proj_z"):
            t = t.view(Hk, 2 * dk + 2 * r * dv, H)
            if part == "in_proj_z":
                return t[:, 2 * dk + r * dv:].reshape(-1, H)
            return torch.cat([t[:, :dk].reshape(-1, H), t[:, dk:2 * dk].reshape(-1, H),
                              t[:, 2 * dk:2 * dk + r * dv].reshape(-1, H)], 0)
        t = t.view(Hk, 2 * r, H)
        return (t[:, :r] if part == "in_proj_b" else t[:, r:]).reshape(-1, H)


def random_weights(cfg: Qwen35Config, seed: int = 0, device="cpu", dtype=torch.bfloat16) -> dict:
    gen = torch.Generator(device=device).manual_seed(seed)
    H = cfg.hidden_size
    w = {}

    def lin(name, o, i, s=1.0):
        w[name] = (torch.randn(o, i, generator=gen, device=device) * s / math.sqrt(i)).to(dtype)

    def vec(name, n, s=0.1, base=0.0):
        w[name] = (base + s * torch.randn(n, generator=gen, device=device)).to(dtype)

    w["model.embed_tokens.weight"] = torch.randn(cfg.vocab_size, H, generator=gen, device=device).to(dtype)
    vec("model.norm.weight", H)
    if not cfg.tie_word_embeddings:
        lin("lm_head.weight", cfg.vocab_size, H)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        vec(p + "input_layernorm.weight", H)
        vec(p + "post_attention_layernorm.weight", H)
        if cfg.is_moe_layer(i):
            m, I, Is = p + "mlp.", cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
            lin(m + "gate.weight", cfg.num_experts, H)
            for e in range(cfg.num_experts):
                lin(m + f"experts.{e}.gate_proj.weight", I, H)
                lin(m + f"experts.{e}.up_proj.weight", I, H)
                lin(m + f"experts.{e}.down_proj.weight", H, I)
            lin(m + "shared_expert.gate_proj.weight", Is, H)
            lin(m + "shared_expert.up_proj.weight", Is, H)
            lin(m + "shared_expert.down_proj.weight", H, Is)
            lin(m + "shared_expert_gate.weight", 1, H)
        else:
            lin(p + "mlp.gate_proj.weight", cfg.intermediate_size, H)
            lin(p + "mlp.up_proj.weight", cfg.intermediate_size, H)
            lin(p + "mlp.down_proj.weight", H, cfg.intermediate_size)
        if cfg.is_linear(i):
            a = p + "linear_attn."
            lin(a + "in_proj_qkv.weight", cfg.conv_dim, H)
            lin(a + "in_proj_z.weight", cfg.value_dim, H)
            lin(a + "in_proj_b.weight", cfg.linear_num_value_heads, H)
            lin(a + "in_proj_a.weight", cfg.linear_num_value_heads, H)
            w[a + "conv1d.weight"] = (torch.randn(cfg.conv_dim, 1, cfg.linear_conv_kernel_dim, generator=gen,
                                                  device=device) * 0.5).to(dtype)
            w[a + "A_log"] = torch.empty(cfg.linear_num_value_heads, device=device).uniform_(
                0, 16, generator=gen).log().to(dtype)
            w[a + "dt_bias"] = torch.ones(cfg.linear_num_value_heads, device=device, dtype=dtype)
            vec(a + "norm.weight", cfg.linear_value_head_dim, base=1.0)
            lin(a + "out_proj.weight", H, cfg.value_dim)
        else:
            a = p + "self_attn."
            nh, nkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
            lin(a + "q_proj.weight", 2 * nh * D, H)
            lin(a + "k_proj.weight", nkv * D, H)
            lin(a + "v_proj.weight", nkv * D, H)
            lin(a + "o_proj.weight", H, nh * D)
            vec(a + "q_norm.weight", D)
            vec(a + "k_norm.weight", D)
    return w


# ---------------------------------------------------------------------------
# fp32 oracle
# ---------------------------------------------------------------------------

class Qwen35Oracle:
    """fp32 full-sequence forward on any device (chunked delta rule)."""

    def __init__(self, cfg: Qwen35Config, weights, device="cpu", chunk: int = 64):
        self.cfg, self.device, self.chunk = cfg, torch.device(device), chunk
        self.w = CanonicalSource(weights, cfg)
        self.inv, self.mult = rope_inv_freq(cfg.rotary_dim, cfg.rope_theta, None, cfg.max_position_embeddings)
        self.inv = self.inv.to(self.device)

    def _t(self, n):
        return self.w[n].to(self.device, torch.float32)

    def _rms(self, x, n, offset=True):
        w = self._t(n) + (1.0 if offset else 0.0)
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps) * w

    def attention(self, i, x, pos):
        from ..ops import reference as R
        c = self.cfg
        a = f"model.layers.{i}.self_attn."
        S, nh, nkv, D = x.shape[0], c.num_attention_heads, c.num_key_value_heads, c.head_dim
        qg = (x @ self._t(a + "q_proj.weight").t()).view(S, nh, 2 * D)
        q, gate = qg[..., :D], qg[..., D:].reshape(S, nh * D)
        k = (x @ self._t(a + "k_proj.weight").t()).view(S, nkv, D)
        v = (x @ self._t(a + "v_proj.weight").t()).view(S, nkv, D)
        q = R.rope(self._rms(q, a + "q_norm.weight"), pos, self.inv, self.mult)
        k = R.rope(self._rms(k, a + "k_norm.weight"), pos, self.inv, self.mult)
        o = R.attention(q, k, v, pos, pos, D ** -0.5, causal=True).reshape(S, nh * D)
        return (o * gate.sigmoid()) @ self._t(a + "o_proj.weight").t()

    def linear_attention(self, i, x, recurrent: bool = False):
        c = self.cfg
        a = f"model.layers.{i}.linear_attn."
        L = x.shape[0]
        Hv, Hk, dk, dv = c.linear_num_value_heads, c.linear_num_key_heads, c.linear_key_head_dim, \
            c.linear_value_head_dim
        mixed = x @ self._t(a + "in_proj_qkv.weight").t()
        z = (x @ self._t(a + "in_proj_z.weight").t()).view(L, Hv, dv)
        gl, beta = gdn_gates(x @ self._t(a + "in_proj_a.weight").t(), x @ self._t(a + "in_proj_b.weight").t(),
                             self._t(a + "A_log"), self._t(a + "dt_bias"))
        y, _ = causal_conv1d(mixed.t(), self._t(a + "conv1d.weight")[:, 0])
        q, k, v = y.t().split([c.key_dim, c.key_dim, c.value_dim], -1)
        rep = Hv // Hk
        q = (l2norm(q.reshape(L, Hk, dk)) * dk ** -0.5).repeat_interleave(rep, 1).transpose(0, 1)
        k = l2norm(k.reshape(L, Hk, dk)).repeat_interleave(rep, 1).transpose(0, 1)
        v = v.reshape(L, Hv, dv).transpose(0, 1)
        fn = gated_delta_recurrent if recurrent else (lambda *t: gated_delta_chunked(*t, chunk=self.chunk))
        o, _ = fn(q, k, v, gl.t(), beta.t())
        o = gated_rmsnorm(o.transpose(0, 1), z, self._t(a + "norm.weight"), c.rms_norm_eps)
        return o.reshape(L, Hv * dv) @ self._t(a + "out_proj.weight").t()

    @torch.no_grad()
    def hidden(self, ids, recurrent: bool = False) -> torch.Tensor:
        c = self.cfg
        ids = torch.as_tensor(ids, device=self.device).long()
        pos = torch.arange(ids.shape[0], device=self.device)
        h = self._t("model.embed_tokens.weight")[ids]
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            x = self._rms(h, p + "input_layernorm.weight")
            h = h + (self.linear_attention(i, x, recurrent) if c.is_linear(i) else self.attention(i, x, pos))
            x = self._rms(h, p + "post_attention_layernorm.weight")
            h = h + (self.moe(i, x) if c.is_moe_layer(i) else self._swiglu(x, p + "mlp."))
        return self._rms(h, "model.norm.weight")

    def _swiglu(self, x, m):
        return (F.silu(x @ self._t(m + "gate_proj.weight").t()) * (x @ self._t(m + "up_proj.weight").t())) \
            @ self._t(m + "down_proj.weight").t()

    def moe(self, i, x):
        from .deepseek import expert_weights
        c = self.cfg
        m = f"model.layers.{i}.mlp."
        probs = (x @ self._t(m + "gate.weight").t()).softmax(-1)
        top, idx = probs.topk(c.num_experts_per_tok, -1)
        if c.norm_topk_prob:
            top = top / top.sum(-1, keepdim=True)
        out = torch.zeros_like(x)
        for e in idx.unique().tolist():
            rows, slot = (idx == e).nonzero(as_tuple=True)
            g, u, d = (t.to(self.device, torch.float32) for t in
                       expert_weights(self.w, f"model.layers.{i}.", e, c.moe_intermediate_size))
            xe = x[rows]
            out.index_add_(0, rows, ((F.silu(xe @ g.t()) * (xe @ u.t())) @ d.t()) * top[rows, slot, None])
        sh = self._swiglu(x, m + "shared_expert.")
        return out + (x @ self._t(m + "shared_expert_gate.weight").t()).sigmoid() * sh

    @torch.no_grad()
    def logits(self, ids, recurrent: bool = False) -> torch.Tensor:
        head = "model.embed_tokens.weight" if self.cfg.tie_word_embeddings else "lm_head.weight"
        return self.hidden(ids, recurrent) @ self._t(head).t()


# ---------------------------------------------------------------------------
# GPU model (engine interface)
# ---------------------------------------------------------------------------

class HybridCache:
    """Paged KV for the full-attention layers plus per-sequence linear-attention
    state: conv windows [n_lin, slots, 2 (position parity), conv_dim, K-1] bf16
    and recurrent states [n_lin, slots, Hv, dk, dv] fp32."""

    def __init__(self, cfg: Qwen35Config, num_blocks: int, num_slots: int, device):
        n_full = sum(not cfg.is_linear(i) for i in range(cfg.num_hidden_layers))
        n_lin = cfg.num_hidden_layers - n_full
        self.paged = PagedKVCache(max(1, n_full), num_blocks, cfg.num_key_value_heads, cfg.head_dim, device)
        self.k, self.v = self.paged.k, self.paged.v
        self.num_slots = num_slots
        self.conv = torch.zeros(n_lin, num_slots, 2, cfg.conv_dim, cfg.linear_conv_kernel_dim - 1,
                                dtype=torch.bfloat16, device=device)
        self.rec = torch.zeros(n_lin, num_slots, cfg.linear_num_value_heads, cfg.linear_key_head_dim,
                               cfg.linear_value_head_dim, dtype=torch.float32, device=device)

    def layer(self, i: int):
        return self.paged.layer(i)


class _Layer:
    __slots__ = ("ln1", "ln2", "w_gu", "wd", "wo", "linear", "idx", "moe",
                 "w_qkvg", "q_norm", "k_norm",
                 "w_in", "conv_w", "A_log", "dt_bias", "norm_w")


class Qwen35LM:
    """Qwen3.5 hybrid decoder on the sm_100a kernels, driven by ``LLMEngine``."""

    stateful = True

    def __init__(self, cfg: Qwen35Config, weights, device="cuda"):
        from .. import ops
        self.cfg, self.device = cfg, torch.device(device)
        c, dev, bf = cfg, self.device, torch.bfloat16
        if c.linear_key_head_dim != c.linear_value_head_dim:
            raise NotImplementedError("Gated DeltaNet decode kernel needs key head dim == value head dim")
        self.hkv, self.D = c.num_key_value_heads, c.head_dim
        self.scale = c.head_dim ** -0.5
        inv, self.rope_mult = rope_inv_freq(c.rotary_dim, c.rope_theta, None, c.max_position_embeddings)
        self.inv_freq = inv.to(dev)
        src = CanonicalSource(weights, c)

        def g(n):
            return src[n].to(dev)

        def dv(t):
            return t.to(dev, bf).contiguous()

        def dvn(t):  # (1 + w) RMSNorm weights
            return dv(t.float() + 1.0)

        self.embed = dv(g("model.embed_tokens.weight"))
        self.norm = dvn(g("model.norm.weight"))
        self.lm_head = self.embed if c.tie_word_embeddings else dv(g("lm_head.weight"))
        nh, nkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        self.layers = []
        n_full = n_lin = 0
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            L = _Layer()
            L.ln1, L.ln2 = dvn(g(p + "input_layernorm.weight")), dvn(g(p + "post_attention_layernorm.weight"))
            L.moe = None
            if c.is_moe_layer(i):
                from .deepseek import expert_weights
                from .moe import pack_experts
                m = p + "mlp."
                ws = [[t.to(dev).float() for t in expert_weights(src, p, e, c.moe_intermediate_size)]
                      for e in range(c.num_experts)]
                L.moe = (g(m + "gate.weight").to(bf).contiguous(), *pack_experts(*zip(*ws)),
                         g(m + "shared_expert_gate.weight").float().contiguous())
                del ws
                L.w_gu = dv(ops.interleave_gate_up(g(m + "shared_expert.gate_proj.weight"),
                                                   g(m + "shared_expert.up_proj.weight")))
                L.wd = dv(g(m + "shared_expert.down_proj.weight"))
            else:
                L.w_gu = dv(ops.interleave_gate_up(g(p + "mlp.gate_proj.weight"), g(p + "mlp.up_proj.weight")))
                L.wd = dv(g(p + "mlp.down_proj.weight"))
            L.linear = c.is_linear(i)
            if L.linear:
                a = p + "linear_attn."
                L.idx, n_lin = n_lin, n_lin + 1
                L.w_in = dv(torch.cat([g(a + "in_proj_qkv.weight"), g(a + "in_proj_z.weight"),
                                       g(a + "in_proj_b.weight"), g(a + "in_proj_a.weight")], 0))
                L.conv_w = g(a + "conv1d.weight").float().reshape(c.conv_dim, -1).contiguous()
                L.A_log = g(a + "A_log").float().contiguous()
                L.dt_bias = g(a + "dt_bias").float().contiguous()
                L.norm_w = g(a + "norm.weight").float().contiguous()
                L.wo = dv(g(a + "out_proj.weight"))
            else:
                a = p + "self_attn."
                L.idx, n_full = n_full, n_full + 1
                qg = g(a + "q_proj.weight").view(nh, 2, D, -1)  # per head: [query rows | gate rows]
                L.w_qkvg = dv(torch.cat([qg[:, 0].reshape(nh * D, -1), g(a + "k_proj.weight"),
                                         g(a + "v_proj.weight"), qg[:, 1].reshape(nh * D, -1)], 0))
                L.q_norm, L.k_norm = dvn(g(a + "q_norm.weight")), dvn(g(a + "k_norm.weight"))
                L.wo = dv(g(a + "o_proj.weight"))
            self.layers.append(L)
        self.n_full = n_full

    # -- engine interface -------------------------------------------------------
    def make_kv_cache(self, num_blocks: int, num_slots: int = 8) -> HybridCache:
        return HybridCache(self.cfg, num_blocks, num_slots, self.device)

    def kv_bytes_per_block(self) -> int:
        return 2 * max(1, self.n_full) * self.hkv * BLOCK_SIZE * self.D * 2

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        from .. import ops
        return ops.linear(x, self.lm_head, out_dtype=torch.float32)

    def forward(self, fb, kv: HybridCache) -> torch.Tensor:
        x = self.forward_hidden(fb, kv)
        if fb.logit_rows is not None:
            x = x.index_select(0, fb.logit_rows)
        return self.logits(x)

    # -- layers ----------------------------------------------------------------
    def _attention(self, L: _Layer, x: torch.Tensor, fb, kv: HybridCache) -> torch.Tensor:
        from .. import ops
        c = self.cfg
        T = x.shape[0]
        nh, nkv, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        qkvg = ops.linear(x, L.w_qkvg)
        w_qkv = (nh + 2 * nkv) * D
        kc, vc = kv.layer(L.idx)
        q = ops.qkv_rope(qkvg[:, :w_qkv], num_q_heads=nh, num_kv_heads=nkv, head_dim=D, positions=fb.positions,
                         inv_freq=self.inv_freq, rope_scale=self.rope_mult, q_norm=L.q_norm, k_norm=L.k_norm,
                         eps=c.rms_norm_eps, slots=fb.slots, k_cache=kc, v_cache=vc, rot_dim=c.rotary_dim)
        o = torch.empty_like(q)
        nd = fb.num_decode
        if nd > 0:
            ops.decode_attention(q[:nd], kc, vc, fb.dec_block_tables, fb.dec_ctx_lens, scale=self.scale, out=o[:nd])
        if T > nd:
            ops.prefill_attention(q[nd:], kc, vc, fb.pre_block_tables, fb.pre_ctx_lens, fb.pre_cu_q, fb.pre_max_q,
                                  scale=self.scale, out=o[nd:])
        return (o.view(T, nh * D).float() * qkvg[:, w_qkv:].float().sigmoid()).to(torch.bfloat16)

    def _gdn(self, L: _Layer, x: torch.Tensor, fb, kv: HybridCache, slots: torch.Tensor) -> torch.Tensor:
        from .. import ops
        from ..ops._ext import ext
        c = self.cfg
        T = x.shape[0]
        p = ops.linear(x, L.w_in)  # [T, conv_dim | z | b | a]
        out = torch.empty(T, c.value_dim, dtype=torch.bfloat16, device=x.device)
        nd = fb.num_decode
        if nd > 0:
            ext().gdn_decode(p[:nd], L.conv_w, L.A_log, L.dt_bias, L.norm_w, kv.conv[L.idx], kv.rec[L.idx],
                             slots[:nd], fb.positions[:nd], out[:nd], c.linear_num_key_heads,
                             c.linear_num_value_heads, c.linear_value_head_dim, c.rms_norm_eps)
            ops._count(1)
        if T > nd:
            self._gdn_prefill(L, p[nd:], fb, kv, slots[nd:], out[nd:])
        return out

    def _gdn_prefill(self, L: _Layer, p: torch.Tensor, fb, kv: HybridCache, slots: torch.Tensor, out: torch.Tensor):
        """Chunked delta rule per prefill sequence; a chunk that starts at
        position 0 starts from zero state, later chunks continue the slot's."""
        c = self.cfg
        Hv, Hk, dk, dv = c.linear_num_value_heads, c.linear_num_key_heads, c.linear_key_head_dim, \
            c.linear_value_head_dim
        C, vd = c.conv_dim, c.value_dim
        cu, ctx, sl = fb.pre_cu_q.tolist(), fb.pre_ctx_lens.tolist(), slots.tolist()
        rep = Hv // Hk
        for s, n_ctx in enumerate(ctx):
            a, b = cu[s], cu[s + 1]
            n = b - a
            start, slot = n_ctx - n, sl[s]
            rows = p[a:b]
            win = kv.conv[L.idx, slot, start & 1] if start > 0 else None
            y, new_win = causal_conv1d(rows[:, :C].t(), L.conv_w, win)
            kv.conv[L.idx, slot, (start + n) & 1] = new_win
            q, k, v = y.t().split([c.key_dim, c.key_dim, vd], -1)
            q = (l2norm(q.float().reshape(n, Hk, dk)) * dk ** -0.5).repeat_interleave(rep, 1).transpose(0, 1)
            k = l2norm(k.float().reshape(n, Hk, dk)).repeat_interleave(rep, 1).transpose(0, 1)
            v = v.float().reshape(n, Hv, dv).transpose(0, 1)
            gl, beta = gdn_gates(rows[:, C + vd + Hv:C + vd + 2 * Hv], rows[:, C + vd:C + vd + Hv], L.A_log,
                                 L.dt_bias)
            state = kv.rec[L.idx, slot] if start > 0 else None
            o, S = gated_delta_chunked(q, k, v, gl.t(), beta.t(), state)
            kv.rec[L.idx, slot] = S
            o = o.transpose(0, 1).to(torch.bfloat16)
            z = rows[:, C:C + vd].reshape(n, Hv, dv)
            out[a:b] = gated_rmsnorm(o, z, L.norm_w, c.rms_norm_eps).reshape(n, vd).to(torch.bfloat16)

    def forward_hidden(self, fb, kv: HybridCache) -> torch.Tensor:
        from .. import ops
        from .decoder import LocalComm
        c = self.cfg
        comm = LocalComm(c.rms_norm_eps)
        slots = fb.seq_slots
        if slots is None:  # direct calls (LLM.logits): sequence i uses slot i
            nseq = fb.num_decode + (0 if fb.pre_ctx_lens is None else fb.pre_ctx_lens.shape[0])
            slots = torch.arange(nseq, dtype=torch.int32, device=self.device)
        h = ops.embedding(fb.input_ids, self.embed)
        x = ops.rmsnorm(h, self.layers[0].ln1, c.rms_norm_eps)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            a = self._gdn(L, x, fb, kv, slots) if L.linear else self._attention(L, x, fb, kv)
            x = comm.rowpar_add_norm(a, L.wo, h, L.ln2)
            nw = self.layers[i + 1].ln1 if i + 1 < n else self.norm
            if L.moe is not None:
                x = self._moe(L, x, h, nw)
                continue
            if x.shape[0] <= ops.ACC_MAX_M:
                gu = ops.swiglu_acc(ops.linear_acc(x, L.w_gu))
            else:
                gu = ops.linear_swiglu(x, L.w_gu)
            x = comm.rowpar_add_norm(gu, L.wd, h, nw)
        return x

    def _moe(self, L: _Layer, x: torch.Tensor, h: torch.Tensor, nw: torch.Tensor) -> torch.Tensor:
        """h += routed experts (MXFP4 grouped GEMM) + sigmoid-gated shared expert;
        returns rmsnorm(h) * nw."""
        from .. import ops
        from .moe import routed_experts, softmax_topk
        c = self.cfg
        router, gu_w, gu_exp, dn_w, dn_exp, sh_gate = L.moe
        experts, weights = softmax_topk(ops.linear(x, router, out_dtype=torch.float32), c.num_experts_per_tok,
                                        c.norm_topk_prob)
        out = routed_experts(x, experts, weights, gu_w, gu_exp, dn_w, dn_exp, c.num_experts, c.moe_intermediate_size)
        sh = ops.linear(ops.linear_swiglu(x, L.w_gu), L.wd)
        h.add_((sh.float() * torch.sigmoid(x.float() @ sh_gate.t())).to(h.dtype))
        return ops.rmsnorm(out, nw, c.rms_norm_eps, residual=h, residual_out=h)
