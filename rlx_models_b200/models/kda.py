"""Kimi Delta Attention (KDA) and the Kimi-Linear decoder (``kimi_linear``).

KDA is the gated delta rule with a decay per KEY CHANNEL (Gated DeltaNet has
one per head). Per head, with state S [Dk, Dv]:

    q, k, v  = silu(short causal conv(x W_q / W_k / W_v))      (depthwise, no bias)
    q       <- l2norm(q) * Dk^-1/2,  k <- l2norm(k)
    g        = -exp(A_log) * softplus(f_b(f_a(x)) + dt_bias)   (log decay, [Dk] per head)
    beta     = sigmoid(b_proj(x))
    S_t      = diag(exp(g_t)) S_{t-1} + k_t u_t^T,   u_t = beta_t (v_t - (diag(exp(g_t)) S_{t-1})^T k_t)
    o_t      = S_t^T q_t
    out      = o_proj(rmsnorm_head(o) * w * sigmoid(g_b(g_a(x))))

Prefill uses the chunked form. Inside a chunk with cumulative log decay G_i
(per channel), E_ij = exp(G_i - G_j) (j <= i, never above 1) and

    (I + A) U = beta (V - (K * exp(G)) S0),   A_ij = beta_i sum_c k_ic k_jc E_ijc  (j < i)
    O = (Q * exp(G)) S0 + [sum_c q_ic k_jc E_ijc]_{j <= i} U
    S1 = exp(G_C) S0 + (K * exp(G_C - G))^T U

(a lower-triangular solve per chunk; every exponent is <= 0, so no chunk size
overflows). Decode runs the KDA instantiation of the Gated DeltaNet decode
kernel (``kda_decode``: conv step, norms, per-channel decay, delta update,
gated output norm in one kernel per layer).

Kimi-Linear interleaves KDA layers (``linear_attn_config.kda_layers``,
1-indexed) with DeepSeek MLA layers that carry no rotary embedding
(``mla_use_nope``), and uses DeepSeek-V3 MoE routing (sigmoid scores, a
correction bias, group-limited top-k, renormalised, scaled) with shared
experts after ``first_k_dense_replace`` dense layers.

Reference: crates/rlx-models-core/src/standard_decoder.rs (KimiLinearSpec
11492-11525, build_kimi_kda 11527-11680, build_kimi_linear_prefill 11682-);
crates/rlx-kimi-k3/src/kda.rs (KDA weights and names).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from .deepseek import DeepseekConfig, DeepseekOracle
from .mamba2 import conv_window

L2_EPS = 1e-6


def kda_gate(a: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor) -> torch.Tensor:
    """Log decay [T, H, D] from the decay logits a [T, H * D], A_log [H], dt_bias [H * D]."""
    H = A_log.numel()
    x = (a.float() + dt_bias.float()).view(a.shape[0], H, -1)
    return -A_log.float().exp().view(1, H, 1) * F.softplus(x)


def kda_recurrent(q, k, v, g, beta, state=None):
    """Token-by-token KDA. q, k [T, H, Dk], v [T, H, Dv], g [T, H, Dk] (log
    decay), beta [T, H], state [H, Dk, Dv] -> (o [T, H, Dv], state)."""
    T, H, Dk = k.shape
    S = torch.zeros(H, Dk, v.shape[-1], dtype=torch.float32, device=v.device) if state is None else state.float()
    out = []
    for t in range(T):
        S = g[t].float().exp()[..., None] * S
        u = beta[t].float()[:, None] * (v[t].float() - torch.einsum("hk,hkv->hv", k[t].float(), S))
        S = S + k[t].float()[..., None] * u[:, None, :]
        out.append(torch.einsum("hk,hkv->hv", q[t].float(), S))
    return torch.stack(out), S


def kda_chunked(q, k, v, g, beta, state=None, chunk: int = 64):
    """The chunked form of ``kda_recurrent`` (same arguments and results)."""
    T, H, Dk = k.shape
    Dv = v.shape[-1]
    dev = v.device
    S = torch.zeros(H, Dk, Dv, dtype=torch.float32, device=dev) if state is None else state.float().clone()
    pad = (-T) % chunk
    # padded steps: no decay, zero key / value / beta, so they leave the state alone
    q, k, v, g = (F.pad(t.float(), (0, 0, 0, 0, 0, pad)).transpose(0, 1) for t in (q, k, v, g))  # [H, T', .]
    beta = F.pad(beta.float(), (0, 0, 0, pad)).transpose(0, 1)  # [H, T']
    N = (T + pad) // chunk
    lower = torch.ones(chunk, chunk, dtype=torch.bool, device=dev).tril()
    strict = lower.clone().fill_diagonal_(False)
    eye = torch.eye(chunk, device=dev)
    out = torch.empty(H, N * chunk, Dv, dtype=torch.float32, device=dev)
    for n in range(N):
        sl = slice(n * chunk, (n + 1) * chunk)
        qc, kc, vc, bc = q[:, sl], k[:, sl], v[:, sl], beta[:, sl]
        G = g[:, sl].cumsum(1)  # [H, C, Dk]
        diff = (G[:, :, None, :] - G[:, None, :, :]).masked_fill(~lower[None, :, :, None], float("-inf"))
        E = diff.exp()  # [H, C, C, Dk], zero above the diagonal
        KK = torch.einsum("hic,hjc,hijc->hij", kc, kc, E)
        QK = torch.einsum("hic,hjc,hijc->hij", qc, kc, E)
        A = (bc[:, :, None] * KK).masked_fill(~strict, 0.0)
        eg = G.exp()
        rhs = bc[..., None] * (vc - torch.einsum("hic,hcv->hiv", kc * eg, S))
        U = torch.linalg.solve_triangular(eye + A, rhs, upper=False)
        out[:, sl] = torch.einsum("hic,hcv->hiv", qc * eg, S) + QK @ U
        gl = G[:, -1]  # [H, Dk]
        S = gl.exp()[..., None] * S + torch.einsum("hjc,hjv->hcv", kc * (gl[:, None] - G).exp(), U)
    return out[:, :T].transpose(0, 1), S


def kda_layer(get, p: str, x: torch.Tensor, H: int, D: int, eps: float, state=None, windows=None, chunk: int = 64):
    """A KDA block on x [T, hidden] (fp32 math) with weights ``get(p + name)``.
    ``state`` [H, D, D] and ``windows`` (q, k, v conv windows [H*D, K-1])
    continue a sequence. Returns (out [T, hidden], state, windows)."""
    T = x.shape[0]
    w = lambda n: get(p + n).to(x.device, torch.float32)  # noqa: E731
    windows = windows or (None, None, None)
    qkv, new_win = [], []
    for name, win in zip(("q", "k", "v"), windows):
        cw = w(f"{name}_conv1d.weight").reshape(H * D, -1)
        y, nw = conv_window((x @ w(f"{name}_proj.weight").t()).t().contiguous(), cw, None, win)
        qkv.append(y.t().reshape(T, H, D))
        new_win.append(nw)
    q, k, v = qkv
    q = q * torch.rsqrt(q.pow(2).sum(-1, keepdim=True) + L2_EPS) * D ** -0.5
    k = k * torch.rsqrt(k.pow(2).sum(-1, keepdim=True) + L2_EPS)
    g = kda_gate((x @ w("f_a_proj.weight").t()) @ w("f_b_proj.weight").t(), w("A_log").reshape(-1),
                 w("dt_bias").reshape(-1))
    beta = torch.sigmoid(x @ w("b_proj.weight").t())
    o, state = kda_chunked(q, k, v, g, beta, state, chunk)
    o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + eps) * w("o_norm.weight")
    gate = torch.sigmoid((x @ w("g_a_proj.weight").t()) @ w("g_b_proj.weight").t()).view(T, H, D)
    return (o * gate).reshape(T, H * D) @ w("o_proj.weight").t(), state, tuple(new_win)


# ---------------------------------------------------------------------------
# Kimi-Linear
# ---------------------------------------------------------------------------

@dataclass
class KimiLinearConfig(DeepseekConfig):
    model_type: str = "kimi_linear"
    kda_layers: list = field(default_factory=list)  # 1-indexed
    kda_num_heads: int = 32
    kda_head_dim: int = 128
    kda_conv_kernel: int = 4
    mla_use_nope: bool = True

    def is_kda(self, i: int) -> bool:
        return (i + 1) in self.kda_layers

    @classmethod
    def from_dict(cls, d: dict) -> "KimiLinearConfig":
        d = dict(d.get("text_config") or d)
        lac = d.get("linear_attn_config") or {}
        ren = {"num_experts": "n_routed_experts", "num_experts_per_token": "num_experts_per_tok",
               "num_shared_experts": "n_shared_experts", "moe_renormalize": "norm_topk_prob",
               "num_expert_group": "n_group"}
        for a, b in ren.items():
            if a in d and b not in d:
                d[b] = d[a]
        if "moe_router_activation_func" in d:
            d["scoring_func"] = d["moe_router_activation_func"]
        d.setdefault("topk_method", "noaux_tc")
        d["model_type"] = "deepseek_v3"  # DeepseekConfig's V3 defaults, then ours
        base = DeepseekConfig.from_dict(d)
        kw = {f: getattr(base, f) for f in DeepseekConfig.__dataclass_fields__}
        kw["model_type"] = "kimi_linear"
        kw["kda_layers"] = list(lac.get("kda_layers", []))
        kw["kda_num_heads"] = int(lac.get("num_heads", cls.kda_num_heads))
        kw["kda_head_dim"] = int(lac.get("head_dim", cls.kda_head_dim))
        kw["kda_conv_kernel"] = int(lac.get("short_conv_kernel_size", cls.kda_conv_kernel))
        kw["mla_use_nope"] = bool(d.get("mla_use_nope", True))
        return cls(**kw)

    @classmethod
    def from_file(cls, path: str) -> "KimiLinearConfig":
        with open(os.path.join(path, "config.json") if os.path.isdir(path) else path) as f:
            return cls.from_dict(json.load(f))


class KimiNames:
    """Kimi-Linear's MoE names (``block_sparse_moe.experts.{e}.w1 / w3 / w2``,
    ``block_sparse_moe.gate``, ``block_sparse_moe.shared_experts``) seen under the
    DeepSeek names (``mlp.experts.{e}.gate_proj / up_proj / down_proj`` ...)."""

    _EXP = {"w1": "gate_proj", "w3": "up_proj", "w2": "down_proj"}

    def __init__(self, weights):
        self.w = weights
        self.map = {}
        for k in weights.keys():
            n = k
            if ".block_sparse_moe." in n:
                n = n.replace(".block_sparse_moe.", ".mlp.")
                parts = n.split(".")
                if len(parts) >= 3 and parts[-2] in self._EXP:
                    parts[-2] = self._EXP[parts[-2]]
                n = ".".join(parts)
            self.map[n] = k

    def keys(self):
        return list(self.map)

    def __contains__(self, name):
        return name in self.map

    def take(self, name, **kw):
        n = self.map[name]
        return self.w.take(n, **kw) if hasattr(self.w, "take") else self.w[n]

    def __getitem__(self, name):
        return self.take(name)


class KimiLinearOracle(DeepseekOracle):
    """fp32 full-sequence Kimi-Linear forward: KDA layers through ``kda_layer``,
    the other layers through the DeepSeek MLA oracle with zero rotary
    frequencies (NoPE), DeepSeek MoE / dense MLPs."""

    def __init__(self, cfg: KimiLinearConfig, weights, device="cpu", chunk: int = 64):
        super().__init__(cfg, KimiNames(weights), device)
        self.chunk = chunk
        if cfg.mla_use_nope:
            self.inv = torch.zeros_like(self.inv)
            self.mult = 1.0

    def attention(self, i: int, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        if not c.is_kda(i):
            return super().attention(i, x, pos)
        get = (lambda n: self.w.take(n))
        out, _, _ = kda_layer(get, f"model.layers.{i}.self_attn.", x, c.kda_num_heads, c.kda_head_dim,
                              c.rms_norm_eps, chunk=self.chunk)
        return out


def random_weights(cfg: KimiLinearConfig, seed: int = 0, dtype=torch.float32) -> dict:
    """Random Kimi-Linear weights under the checkpoint's names."""
    g = torch.Generator().manual_seed(seed)
    Hd, V = cfg.hidden_size, cfg.vocab_size
    w = {}

    def t(name, *shape, std=0.05):
        w[name] = (torch.randn(*shape, generator=g) * std).to(dtype)

    def ones(name, n):
        w[name] = (1.0 + 0.1 * torch.randn(n, generator=g)).to(dtype)

    t("model.embed_tokens.weight", V, Hd, std=0.5)
    ones("model.norm.weight", Hd)
    t("lm_head.weight", V, Hd)
    nh, dn, dr, dv, r = (cfg.num_attention_heads, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim,
                         cfg.kv_lora_rank)
    H, D, K = cfg.kda_num_heads, cfg.kda_head_dim, cfg.kda_conv_kernel
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        ones(p + "input_layernorm.weight", Hd)
        ones(p + "post_attention_layernorm.weight", Hd)
        a = p + "self_attn."
        if cfg.is_kda(i):
            for n in ("q", "k", "v"):
                t(a + f"{n}_proj.weight", H * D, Hd, std=0.2)
                t(a + f"{n}_conv1d.weight", H * D, 1, K, std=0.5)
            t(a + "f_a_proj.weight", D, Hd, std=0.2)
            t(a + "f_b_proj.weight", H * D, D, std=0.3)
            t(a + "g_a_proj.weight", D, Hd, std=0.2)
            t(a + "g_b_proj.weight", H * D, D, std=0.3)
            t(a + "b_proj.weight", H, Hd, std=0.3)
            w[a + "A_log"] = torch.empty(H).uniform_(0.0, 2.0, generator=g).log().to(dtype)
            t(a + "dt_bias", H * D, std=0.5)
            ones(a + "o_norm.weight", D)
            t(a + "o_proj.weight", Hd, H * D)
        else:
            t(a + "q_proj.weight", nh * (dn + dr), Hd)
            t(a + "kv_a_proj_with_mqa.weight", r + dr, Hd)
            ones(a + "kv_a_layernorm.weight", r)
            t(a + "kv_b_proj.weight", nh * (dn + dv), r)
            t(a + "o_proj.weight", Hd, nh * dv)
        if cfg.is_moe(i):
            m = p + "block_sparse_moe."
            t(m + "gate.weight", cfg.n_routed_experts, Hd)
            w[m + "gate.e_score_correction_bias"] = (0.1 * torch.randn(cfg.n_routed_experts, generator=g)).float()
            for e in range(cfg.n_routed_experts):
                for n, shape in (("w1", (cfg.moe_intermediate_size, Hd)), ("w3", (cfg.moe_intermediate_size, Hd)),
                                 ("w2", (Hd, cfg.moe_intermediate_size))):
                    t(m + f"experts.{e}.{n}.weight", *shape)
            si = cfg.moe_intermediate_size * (cfg.n_shared_experts or 0)
            if si:
                t(m + "shared_experts.gate_proj.weight", si, Hd)
                t(m + "shared_experts.up_proj.weight", si, Hd)
                t(m + "shared_experts.down_proj.weight", Hd, si)
        else:
            t(p + "mlp.gate_proj.weight", cfg.intermediate_size, Hd)
            t(p + "mlp.up_proj.weight", cfg.intermediate_size, Hd)
            t(p + "mlp.down_proj.weight", Hd, cfg.intermediate_size)
    return w
