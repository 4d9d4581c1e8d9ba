"""DeepSeek-V2 / V3 family (Kimi-K2 is the V3 architecture): multi-head
latent attention (MLA) and DeepSeekMoE, served through the paged engine.

MLA per layer (HF names):

    q    = q_b(rms(q_a(x)))  or  q_proj(x)          -> [T, nh, nope + rope]
    ckv  = kv_a_proj_with_mqa(x) = [c (kv_lora) | k_rope (one shared head)]
    k, v = kv_b(rms(c)) split per head into [nope | v]
    RoPE on the rope slices only (pairs (2i, 2i+1) when ``rope_interleave``)
    score scale = qk_head_dim^-0.5 x yarn_mscale(factor, mscale_all_dim)^2

B200 layout: the paged cache holds only the latent row [rms(c) | rope(k_rope)]
(kv_lora + rope values per token per layer, 576 for V3, against
2 x nh x 192 = 49152 for the expanded K/V), one page of 16 tokens contiguous.
``q_a_proj`` and ``kv_a_proj_with_mqa`` run as one GEMM (x is read once).
Decode attention is the absorbed form: q_nope is mapped into the latent space
through kv_b's key half (q_lat = q_nope W_UK, per head), scores are
[q_lat | q_rope] . [c | k_rope] over the latent rows (a multi-query attention
with a 576-wide head shared by all heads), the probabilities weight the
latent rows, and kv_b's value half maps the result back (o = (P c) W_UV).
Prefill expands the context's latent rows through kv_b (cheaper per query
when many queries share the keys) and runs causal attention per sequence.

DeepSeekMoE: router logits in fp32; scores sigmoid (V3, with the per-expert
``e_score_correction_bias`` added for the choice only) or softmax (V2);
group-limited choice (V3 "noaux_tc": a group's score is the sum of its top-2;
V2 "group_limited_greedy": its max; ``topk_group`` groups survive); top-k;
weights taken from the un-biased scores, normalised when ``norm_topk_prob``,
times ``routed_scaling_factor``. Routed experts run on the grouped MXFP4 GEMM
(weights packed at load); the ``n_shared_experts`` shared expert is a dense
SwiGLU on the tcgen05 GEMM; the first ``first_k_dense_replace`` layers are
dense.

GLM-4.7-Flash (``glm4_moe_lite``) is this architecture with GLM-4.5's router
and per-layer ``mlp_layer_types``; GLM-5 (``glm_moe_dsa``) adds DeepSeek
sparse attention: an indexer (its own small multi-head projections from the
q_a latent and the hidden state, ReLU scores weighted per head) keeps the
``index_topk`` best keys per query, and RoPE rotates split halves. The oracle
applies the indexer; the served model attends densely, which is the same
model while a sequence holds at most ``index_topk`` (2048) tokens.

``DeepseekOracle`` is the fp32 full-sequence restatement (expanded MLA, exact
routing); it matches ``transformers``' DeepseekV3 / V2 on CPU and is the GPU
model's numerics reference.

Reference: crates/rlx-deepseek/src/config.rs:35-150 (`DeepseekV3Config`,
`is_moe_layer`, `attn_score_scale`), src/mla.rs:16-30 and :84-194
(`emit_mla_attention`: the same projections, expanded K/V with the value
zero-padded to the qk width), src/moe.rs:16-40 and :133-279
(`emit_deepseek_moe`: noaux_tc group-limited router, shared expert);
rlx-models-core src/standard_decoder.rs:2045 (`build_deepseek_mla`);
crates/rlx-glm5next src/indexer.rs (DSA indexer), src/mla.rs.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass, field, fields

import torch
import torch.nn.functional as F

from ..ops import rope_inv_freq
from ..runtime.kv_cache import BLOCK_SIZE

DEEPSEEK_TYPES = ("deepseek_v3", "deepseek_v2", "kimi_k2", "glm4_moe_lite", "glm_moe_dsa")
_SUB_NORM_EPS = 1e-6  # q_a_layernorm / kv_a_layernorm use the RMSNorm default, not rms_norm_eps


@dataclass
class DeepseekConfig:
    model_type: str = "deepseek_v3"
    vocab_size: int = 129280
    hidden_size: int = 7168
    intermediate_size: int = 18432
    moe_intermediate_size: int = 2048
    num_hidden_layers: int = 61
    num_attention_heads: int = 128
    n_shared_experts: int | None = 1
    n_routed_experts: int | None = 256
    routed_scaling_factor: float = 2.5
    kv_lora_rank: int = 512
    q_lora_rank: int | None = 1536
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    qk_nope_head_dim: int = 128
    n_group: int = 8
    topk_group: int = 4
    num_experts_per_tok: int = 8
    first_k_dense_replace: int = 3
    moe_layer_freq: int = 1
    norm_topk_prob: bool = True
    scoring_func: str = "sigmoid"
    topk_method: str = "noaux_tc"
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: dict | None = None
    rope_interleave: bool = True
    max_position_embeddings: int = 4096
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    bos_token_id: int | None = 0
    eos_token_id: int | list | None = 1
    mlp_layer_types: list | None = None  # GLM: "dense" / "sparse" per layer (overrides first_k_dense_replace)
    index_topk: int = 0  # GLM-5 DSA: keys kept per query by the indexer (0: dense attention)
    index_n_heads: int = 32
    index_head_dim: int = 128
    extra: dict = field(default_factory=dict)

    @property
    def qk_head_dim(self) -> int:
        return self.qk_nope_head_dim + self.qk_rope_head_dim

    @property
    def latent_dim(self) -> int:
        return self.kv_lora_rank + self.qk_rope_head_dim

    def is_moe(self, i: int) -> bool:
        if self.mlp_layer_types:
            return bool(self.n_routed_experts) and self.mlp_layer_types[i] == "sparse"
        return bool(self.n_routed_experts) and i >= self.first_k_dense_replace and i % self.moe_layer_freq == 0

    @property
    def softmax_scale(self) -> float:
        s = self.qk_head_dim ** -0.5
        r = self.rope_scaling or {}
        kind = r.get("rope_type", r.get("type", "default"))
        if kind not in (None, "default") and r.get("mscale_all_dim") and float(r.get("factor", 1.0)) > 1.0:
            m = 0.1 * float(r["mscale_all_dim"]) * math.log(float(r["factor"])) + 1.0
            s *= m * m
        return s

    @classmethod
    def from_dict(cls, d: dict) -> "DeepseekConfig":
        d = dict(d)
        mt = d.get("model_type", "deepseek_v3")
        kw = {f.name: d[f.name] for f in fields(cls) if f.name in d and f.name != "extra"}
        rp = d.get("rope_parameters") or d.get("rope_scaling")
        if rp:
            rp = dict(rp)
            if "rope_theta" in rp:
                kw["rope_theta"] = float(rp.pop("rope_theta"))
            kind = rp.get("rope_type", rp.get("type", "default"))
            kw["rope_scaling"] = None if kind in (None, "default") else rp
        if mt == "deepseek_v2":  # V2 defaults differ from V3's
            kw.setdefault("scoring_func", "softmax")
            kw.setdefault("topk_method", "greedy")
            kw.setdefault("first_k_dense_replace", 0)
            kw.setdefault("norm_topk_prob", False)
            kw.setdefault("routed_scaling_factor", 1.0)
            kw.setdefault("rope_interleave", True)
        if mt in ("glm4_moe_lite", "glm_moe_dsa"):  # GLM-4.7-Flash / GLM-5: MLA + GLM-4.5's MoE
            n = kw.get("num_hidden_layers", cls.num_hidden_layers)
            if not kw.get("mlp_layer_types"):
                k0 = 1 if mt == "glm4_moe_lite" else min(3, n)
                kw["mlp_layer_types"] = ["dense"] * k0 + ["sparse"] * (n - k0)
            kw.setdefault("rms_norm_eps", 1e-5)
            kw.setdefault("routed_scaling_factor", 1.8 if mt == "glm4_moe_lite" else 2.5)
            for k in ("n_group", "topk_group"):
                kw.setdefault(k, 1)
            if mt == "glm_moe_dsa":
                kw["rope_interleave"] = False  # GLM-5 rotates split halves in MLA and the indexer
                kw.setdefault("index_topk", 2048)
            else:
                kw["index_topk"] = 0
        for k in ("n_group", "topk_group"):
            if kw.get(k) is None:
                kw[k] = 1
        return cls(**kw)

    @classmethod
    def from_file(cls, path: str) -> "DeepseekConfig":
        with open(os.path.join(path, "config.json") if os.path.isdir(path) else path) as f:
            return cls.from_dict(json.load(f))

    def to_hf_dict(self) -> dict:
        d = {f.name: getattr(self, f.name) for f in fields(self) if f.name not in ("extra", "rope_scaling")}
        rp = {"rope_type": "default", "rope_theta": self.rope_theta}
        if self.rope_scaling:
            rp = dict(self.rope_scaling, rope_theta=self.rope_theta)
        d["rope_parameters"] = rp
        return d


def is_deepseek_config(path: str) -> bool:
    p = os.path.join(path, "config.json") if os.path.isdir(path) else path
    try:
        with open(p) as f:
            return json.load(f).get("model_type") in DEEPSEEK_TYPES
    except (OSError, ValueError):
        return False


# ---------------------------------------------------------------------------
# shared math (oracle and GPU model)
# ---------------------------------------------------------------------------

def rope_tables(cfg: DeepseekConfig, device) -> tuple[torch.Tensor, float]:
    inv, mult = rope_inv_freq(cfg.qk_rope_head_dim, cfg.rope_theta, cfg.rope_scaling, cfg.max_position_embeddings)
    return inv.to(device), float(mult)


def apply_rope(x: torch.Tensor, pos: torch.Tensor, inv: torch.Tensor, mult: float, interleave: bool) -> torch.Tensor:
    """x [T, ..., d] (d = rope dim), pos [T]. Rotates pair i by pos * inv[i];
    pairs are (2i, 2i+1) when ``interleave`` else (i, i + d/2). The result is
    in split layout [rotated firsts | rotated seconds] either way (the dot
    products of q and k, rotated alike, do not depend on the layout)."""
    xf = x.float()
    ang = pos.float()[:, None] * inv[None, :]
    shape = (x.shape[0],) + (1,) * (x.dim() - 2) + (inv.shape[0],)
    cos, sin = (ang.cos() * mult).view(shape), (ang.sin() * mult).view(shape)
    if interleave:
        x1, x2 = xf[..., 0::2], xf[..., 1::2]
    else:
        h = x.shape[-1] // 2
        x1, x2 = xf[..., :h], xf[..., h:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).to(x.dtype)


def route(cfg: DeepseekConfig, logits: torch.Tensor, bias: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 router logits [T, E] -> (expert ids [T, k] int64, weights [T, k] fp32)."""
    T, E = logits.shape
    scores = logits.sigmoid() if cfg.scoring_func == "sigmoid" else logits.softmax(-1)
    choice = scores + bias if bias is not None else scores
    if cfg.topk_method in ("noaux_tc", "group_limited_greedy") and cfg.n_group > 1:
        g = choice.view(T, cfg.n_group, E // cfg.n_group)
        gs = g.topk(2, -1)[0].sum(-1) if cfg.topk_method == "noaux_tc" else g.amax(-1)
        keep = torch.zeros_like(gs).scatter_(1, gs.topk(cfg.topk_group, -1)[1], 1.0)
        choice = choice.masked_fill(~keep.bool()[..., None].expand_as(g).reshape(T, E), 0.0)
    idx = choice.topk(cfg.num_experts_per_tok, -1)[1]
    w = scores.gather(1, idx)
    if cfg.norm_topk_prob:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return idx, w * cfg.routed_scaling_factor


def _getter(weights):
    return (lambda n: weights.take(n)) if hasattr(weights, "take") else (lambda n: weights[n])


def expert_weights(weights, prefix: str, e: int, inter: int):
    """(gate [I, H], up [I, H], down [H, I]) of routed expert ``e`` from either
    checkpoint layout: per-expert ``experts.{e}.*_proj.weight`` (the released
    checkpoints) or fused ``experts.gate_up_proj`` [E, 2I, H] / ``experts.down_proj``
    [E, H, I] (transformers' in-memory layout)."""
    g = _getter(weights)
    pe = prefix + "mlp.experts."
    if (pe + f"{e}.gate_proj.weight") in weights:
        return g(pe + f"{e}.gate_proj.weight"), g(pe + f"{e}.up_proj.weight"), g(pe + f"{e}.down_proj.weight")
    gu = g(pe + "gate_up_proj")[e]
    return gu[:inter], gu[inter:], g(pe + "down_proj")[e]


def random_weights(cfg: DeepseekConfig, seed: int = 0, device="cpu", dtype=torch.bfloat16) -> dict:
    """Seeded random weights with the released checkpoints' tensor names."""
    gen = torch.Generator(device=device).manual_seed(seed)
    H, nh = cfg.hidden_size, cfg.num_attention_heads
    w = {}

    def lin(name, o, i):
        w[name] = (torch.randn(o, i, generator=gen, device=device) / math.sqrt(i)).to(dtype)

    def ones(name, n):
        w[name] = torch.ones(n, device=device, dtype=dtype)

    w["model.embed_tokens.weight"] = (torch.randn(cfg.vocab_size, H, generator=gen, device=device) * 0.5).to(dtype)
    ones("model.norm.weight", H)
    if not cfg.tie_word_embeddings:
        lin("lm_head.weight", cfg.vocab_size, H)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        ones(p + "input_layernorm.weight", H)
        ones(p + "post_attention_layernorm.weight", H)
        a = p + "self_attn."
        if cfg.q_lora_rank:
            lin(a + "q_a_proj.weight", cfg.q_lora_rank, H)
            ones(a + "q_a_layernorm.weight", cfg.q_lora_rank)
            lin(a + "q_b_proj.weight", nh * cfg.qk_head_dim, cfg.q_lora_rank)
        else:
            lin(a + "q_proj.weight", nh * cfg.qk_head_dim, H)
        lin(a + "kv_a_proj_with_mqa.weight", cfg.latent_dim, H)
        ones(a + "kv_a_layernorm.weight", cfg.kv_lora_rank)
        lin(a + "kv_b_proj.weight", nh * (cfg.qk_nope_head_dim + cfg.v_head_dim), cfg.kv_lora_rank)
        lin(a + "o_proj.weight", H, nh * cfg.v_head_dim)
        if cfg.index_topk and cfg.q_lora_rank:
            x = a + "indexer."
            lin(x + "wq_b.weight", cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank)
            lin(x + "wk.weight", cfg.index_head_dim, H)
            ones(x + "k_norm.weight", cfg.index_head_dim)
            w[x + "k_norm.bias"] = torch.zeros(cfg.index_head_dim, device=device, dtype=dtype)
            lin(x + "weights_proj.weight", cfg.index_n_heads, H)
        m = p + "mlp."
        if cfg.is_moe(i):
            I = cfg.moe_intermediate_size
            lin(m + "gate.weight", cfg.n_routed_experts, H)
            if cfg.topk_method == "noaux_tc":
                w[m + "gate.e_score_correction_bias"] = (torch.randn(cfg.n_routed_experts, generator=gen,
                                                                     device=device) * 0.1).float()
            for e in range(cfg.n_routed_experts):
                lin(m + f"experts.{e}.gate_proj.weight", I, H)
                lin(m + f"experts.{e}.up_proj.weight", I, H)
                lin(m + f"experts.{e}.down_proj.weight", H, I)
            if cfg.n_shared_experts:
                Is = I * cfg.n_shared_experts
                lin(m + "shared_experts.gate_proj.weight", Is, H)
                lin(m + "shared_experts.up_proj.weight", Is, H)
                lin(m + "shared_experts.down_proj.weight", H, Is)
        else:
            lin(m + "gate_proj.weight", cfg.intermediate_size, H)
            lin(m + "up_proj.weight", cfg.intermediate_size, H)
            lin(m + "down_proj.weight", H, cfg.intermediate_size)
    return w


# ---------------------------------------------------------------------------
# fp32 oracle
# ---------------------------------------------------------------------------

class DeepseekOracle:
    """fp32 full-sequence forward (expanded MLA, exact routing) on any device."""

    def __init__(self, cfg: DeepseekConfig, weights, device="cpu"):
        self.cfg, self.w, self.device = cfg, weights, torch.device(device)
        self.inv, self.mult = rope_tables(cfg, self.device)

    def _t(self, name):
        return _getter(self.w)(name).to(self.device, torch.float32)

    @staticmethod
    def _rms(x, w, eps):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w

    def _mlp(self, x, p):
        g, u, d = (self._t(p + n + "_proj.weight") for n in ("gate", "up", "down"))
        return (F.silu(x @ g.t()) * (x @ u.t())) @ d.t()

    def attention(self, i: int, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        return self.attention_heads(i, x, pos) @ self._t(f"model.layers.{i}.self_attn.o_proj.weight").t()

    def attention_heads(self, i: int, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Causal MLA of layer ``i`` before o_proj: [S, nh * v_head_dim]."""
        c = self.cfg
        S = x.shape[0]
        nh, dn, dr, dv, r = c.num_attention_heads, c.qk_nope_head_dim, c.qk_rope_head_dim, c.v_head_dim, c.kv_lora_rank
        a = f"model.layers.{i}.self_attn."
        q_res = None
        if c.q_lora_rank:
            q_res = self._rms(x @ self._t(a + "q_a_proj.weight").t(), self._t(a + "q_a_layernorm.weight"),
                              _SUB_NORM_EPS)
            q = q_res @ self._t(a + "q_b_proj.weight").t()
        else:
            q = x @ self._t(a + "q_proj.weight").t()
        q = q.view(S, nh, dn + dr)
        ckv = x @ self._t(a + "kv_a_proj_with_mqa.weight").t()
        kv = self._rms(ckv[:, :r], self._t(a + "kv_a_layernorm.weight"), _SUB_NORM_EPS) @ \
            self._t(a + "kv_b_proj.weight").t()
        kv = kv.view(S, nh, dn + dv)
        q_rot = apply_rope(q[..., dn:], pos, self.inv, self.mult, c.rope_interleave)
        k_rot = apply_rope(ckv[:, None, r:], pos, self.inv, self.mult, c.rope_interleave).expand(S, nh, dr)
        qf = torch.cat([q[..., :dn], q_rot], -1).transpose(0, 1)
        kf = torch.cat([kv[..., :dn], k_rot], -1).transpose(0, 1)
        mask = None
        if c.index_topk and q_res is not None and (a + "indexer.wq_b.weight") in self.w:
            sel = self.dsa_select(i, x, q_res, pos)
            mask = torch.zeros(S, S, dtype=torch.bool, device=x.device).scatter_(1, sel, True)
            mask &= torch.ones(S, S, dtype=torch.bool, device=x.device).tril()
        o = F.scaled_dot_product_attention(qf, kf, kv[..., dn:].transpose(0, 1), attn_mask=mask,
                                           is_causal=mask is None, scale=c.softmax_scale)
        return o.transpose(0, 1).reshape(S, nh * dv)

    def dsa_select(self, i: int, x: torch.Tensor, q_res: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """GLM-5 DSA indexer of layer ``i``: [S, min(index_topk, S)] key positions
        per query. Index queries come from the normalised q_a latent, one index
        key per token (LayerNorm of wk(x)); both carry RoPE on their first
        qk_rope_head_dim values. score[s, t] = sum_h w[s, h] relu(q[s, h] . k[t] / sqrt(D)),
        w = weights_proj(x) / sqrt(heads); future positions score -inf."""
        c = self.cfg
        a = f"model.layers.{i}.self_attn.indexer."
        S, H, D, dr = x.shape[0], c.index_n_heads, c.index_head_dim, c.qk_rope_head_dim
        q = (q_res @ self._t(a + "wq_b.weight").t()).view(S, H, D)
        k = F.layer_norm(x @ self._t(a + "wk.weight").t(), (D,), self._t(a + "k_norm.weight"),
                         self._t(a + "k_norm.bias"), 1e-6)
        q = torch.cat([apply_rope(q[..., :dr], pos, self.inv, self.mult, False), q[..., dr:]], -1)
        k = torch.cat([apply_rope(k[:, None, :dr], pos, self.inv, self.mult, False)[:, 0], k[:, dr:]], -1)
        w = (x @ self._t(a + "weights_proj.weight").t()) * H ** -0.5
        score = torch.einsum("sht,sh->st", torch.relu(torch.einsum("shd,td->sht", q, k) * D ** -0.5), w)
        future = torch.ones(S, S, dtype=torch.bool, device=x.device).triu(1)
        return score.masked_fill(future, float("-inf")).topk(min(c.index_topk, S), -1).indices

    def moe(self, i: int, x: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        p = f"model.layers.{i}.mlp."
        bias = self._t(p + "gate.e_score_correction_bias") if (p + "gate.e_score_correction_bias") in self.w else None
        idx, wts = route(c, x @ self._t(p + "gate.weight").t(), bias)
        out = torch.zeros_like(x)
        for e in idx.unique().tolist():
            rows, slot = (idx == e).nonzero(as_tuple=True)
            g, u, d = (t.to(self.device, torch.float32) for t in
                       expert_weights(self.w, f"model.layers.{i}.", e, c.moe_intermediate_size))
            xe = x[rows]
            out.index_add_(0, rows, ((F.silu(xe @ g.t()) * (xe @ u.t())) @ d.t()) * wts[rows, slot, None])
        if c.n_shared_experts:
            out = out + self._mlp(x, p + "shared_experts.")
        return out

    @torch.no_grad()
    def hidden(self, ids) -> torch.Tensor:
        c = self.cfg
        ids = torch.as_tensor(ids, device=self.device).long()
        pos = torch.arange(ids.shape[0], device=self.device)
        h = self._t("model.embed_tokens.weight")[ids]
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            h = h + self.attention(i, self._rms(h, self._t(p + "input_layernorm.weight"), c.rms_norm_eps), pos)
            x = self._rms(h, self._t(p + "post_attention_layernorm.weight"), c.rms_norm_eps)
            h = h + (self.moe(i, x) if c.is_moe(i) else self._mlp(x, p + "mlp."))
        return self._rms(h, self._t("model.norm.weight"), c.rms_norm_eps)

    @torch.no_grad()
    def logits(self, ids) -> torch.Tensor:
        head = "model.embed_tokens.weight" if self.cfg.tie_word_embeddings else "lm_head.weight"
        return self.hidden(ids) @ self._t(head).t()


def latent_decode_attention(q_nope: torch.Tensor, q_rope: torch.Tensor, w_uk: torch.Tensor, w_uv_t: torch.Tensor,
                            cache: torch.Tensor, tables: torch.Tensor, ctx_lens: torch.Tensor,
                            scale: float) -> torch.Tensor:
    """Absorbed MLA decode over a paged latent cache.

    q_nope [B, nh, dn], q_rope [B, nh, dr] (rotated), w_uk [nh, dn, r] and
    w_uv_t [nh, r, dv] (kv_b's key / value halves), cache [blocks, 16, r + dr],
    tables [B, W] block ids, ctx_lens [B] -> [B, nh * dv]."""
    B, nh, _ = q_nope.shape
    r = w_uk.shape[2]
    q_lat = torch.bmm(q_nope.transpose(0, 1), w_uk).transpose(0, 1)  # [B, nh, r]
    qf = torch.cat([q_lat, q_rope.to(q_lat.dtype)], -1)
    W = tables.shape[1]
    lat = cache[tables.long()].reshape(B, W * BLOCK_SIZE, cache.shape[-1])  # [B, S, r + dr]
    s = torch.bmm(qf, lat.transpose(1, 2)).float() * scale  # [B, nh, S]
    valid = torch.arange(W * BLOCK_SIZE, device=s.device)[None, :] < ctx_lens.to(s.device).long()[:, None]
    s = s.masked_fill(~valid[:, None, :], float("-inf"))
    p = s.softmax(-1).to(lat.dtype)
    o = torch.bmm(p, lat[..., :r])  # [B, nh, r]
    o = torch.bmm(o.transpose(0, 1), w_uv_t)  # [nh, B, dv]
    return o.transpose(0, 1).reshape(B, -1)


# ---------------------------------------------------------------------------
# GPU model (engine interface)
# ---------------------------------------------------------------------------

class MLACache:
    """Paged latent cache: [layers, blocks, 16, kv_lora + rope] bf16."""

    def __init__(self, num_layers: int, num_blocks: int, width: int, device):
        self.num_layers, self.num_blocks, self.width = num_layers, num_blocks, width
        self.k = torch.zeros(num_layers, num_blocks, BLOCK_SIZE, width, dtype=torch.bfloat16, device=device)
        self.v = None

    def layer(self, i: int):
        return self.k[i], None


class _Layer:
    __slots__ = ("ln1", "ln2", "w_a", "q_ln", "q_b", "kv_ln", "w_kvb", "w_uk", "w_uv_t", "wo",
                 "w_gu", "wd", "moe")


class _MoE:
    __slots__ = ("router_w", "router_b", "gu_w", "gu_exp", "dn_w", "dn_exp", "sh_gu", "sh_dn")


class DeepseekLM:
    """MLA + DeepSeekMoE decoder on the sm_100a kernels, driven by ``LLMEngine``."""

    def __init__(self, cfg: DeepseekConfig, weights, device="cuda"):
        from .. import ops
        from .moe import pack_experts
        if cfg.index_topk:
            import warnings
            warnings.warn(f"{cfg.model_type}: the served model attends densely; it equals the DSA model while a "
                          f"sequence holds at most index_topk={cfg.index_topk} tokens")
        self.cfg, self.device = cfg, torch.device(device)
        self.hkv, self.D = 1, cfg.latent_dim  # one shared latent "head" per token
        c, dev, bf = cfg, self.device, torch.bfloat16
        g = _getter(weights)

        def dv(t):
            return t.to(device=dev, dtype=bf).contiguous()

        self.embed = dv(g("model.embed_tokens.weight"))
        self.norm = dv(g("model.norm.weight"))
        self.lm_head = self.embed if c.tie_word_embeddings else dv(g("lm_head.weight"))
        self.inv, self.mult = rope_tables(c, dev)
        nh, dn, dv_, r = c.num_attention_heads, c.qk_nope_head_dim, c.v_head_dim, c.kv_lora_rank
        self.layers = []
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            a = p + "self_attn."
            L = _Layer()
            L.ln1, L.ln2 = dv(g(p + "input_layernorm.weight")), dv(g(p + "post_attention_layernorm.weight"))
            qw = g(a + "q_a_proj.weight") if c.q_lora_rank else g(a + "q_proj.weight")
            L.w_a = dv(torch.cat([qw.to(dev), g(a + "kv_a_proj_with_mqa.weight").to(dev)], 0))
            L.q_ln = dv(g(a + "q_a_layernorm.weight")) if c.q_lora_rank else None
            L.q_b = dv(g(a + "q_b_proj.weight")) if c.q_lora_rank else None
            L.kv_ln = dv(g(a + "kv_a_layernorm.weight"))
            L.w_kvb = dv(g(a + "kv_b_proj.weight"))
            kvb = L.w_kvb.view(nh, dn + dv_, r)
            L.w_uk = kvb[:, :dn].contiguous()  # [nh, dn, r]
            L.w_uv_t = kvb[:, dn:].transpose(1, 2).contiguous()  # [nh, r, dv]
            L.wo = dv(g(a + "o_proj.weight"))
            L.w_gu = L.wd = L.moe = None
            m = p + "mlp."
            if c.is_moe(i):
                M = _MoE()
                M.router_w = g(m + "gate.weight").to(dev, torch.float32).contiguous()
                bn = m + "gate.e_score_correction_bias"
                M.router_b = g(bn).to(dev, torch.float32) if bn in weights else None
                I = c.moe_intermediate_size
                ws = [[t.to(dev).float() for t in expert_weights(weights, p, e, I)] for e in range(c.n_routed_experts)]
                M.gu_w, M.gu_exp, M.dn_w, M.dn_exp = pack_experts(*zip(*ws))
                del ws
                M.sh_gu = M.sh_dn = None
                if c.n_shared_experts:
                    s = m + "shared_experts."
                    M.sh_gu = dv(ops.interleave_gate_up(g(s + "gate_proj.weight").to(dev), g(s + "up_proj.weight").to(dev)))
                    M.sh_dn = dv(g(s + "down_proj.weight"))
                L.moe = M
            else:
                L.w_gu = dv(ops.interleave_gate_up(g(m + "gate_proj.weight").to(dev), g(m + "up_proj.weight").to(dev)))
                L.wd = dv(g(m + "down_proj.weight"))
            self.layers.append(L)

    # -- engine interface -------------------------------------------------------
    def make_kv_cache(self, num_blocks: int) -> MLACache:
        return MLACache(self.cfg.num_hidden_layers, num_blocks, self.cfg.latent_dim, self.device)

    def kv_bytes_per_block(self) -> int:
        return self.cfg.num_hidden_layers * BLOCK_SIZE * self.cfg.latent_dim * 2

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        from .. import ops
        return ops.linear(x, self.lm_head, out_dtype=torch.float32)

    def forward(self, fb, kv: MLACache) -> torch.Tensor:
        x = self.forward_hidden(fb, kv)
        if fb.logit_rows is not None:
            x = x.index_select(0, fb.logit_rows)
        return self.logits(x)

    # -- layers ----------------------------------------------------------------
    def _mla(self, i: int, L: _Layer, x: torch.Tensor, fb, kv: MLACache) -> torch.Tensor:
        from .. import ops
        c = self.cfg
        T = x.shape[0]
        nh, dn, dr, dv, r = c.num_attention_heads, c.qk_nope_head_dim, c.qk_rope_head_dim, c.v_head_dim, c.kv_lora_rank
        a = ops.linear(x, L.w_a)  # [T, (q_lora | nh*qk) + r + dr]: q_a and kv_a in one GEMM
        nq = a.shape[1] - c.latent_dim
        if c.q_lora_rank:
            q = ops.linear(ops.rmsnorm(a[:, :nq].contiguous(), L.q_ln, _SUB_NORM_EPS), L.q_b)
        else:
            q = a[:, :nq]
        q = q.reshape(T, nh, dn + dr)
        pos = fb.positions
        q_rope = apply_rope(q[..., dn:], pos, self.inv, self.mult, c.rope_interleave)
        k_rope = apply_rope(a[:, nq + r:], pos, self.inv, self.mult, c.rope_interleave)
        lat = torch.cat([ops.rmsnorm(a[:, nq:nq + r].contiguous(), L.kv_ln, _SUB_NORM_EPS), k_rope], -1)
        cache = kv.k[i]
        cache.view(-1, c.latent_dim).index_copy_(0, fb.slots, lat)
        out = torch.empty(T, nh * dv, dtype=torch.bfloat16, device=x.device)
        nd = fb.num_decode
        if nd > 0:
            out[:nd] = latent_decode_attention(q[:nd, :, :dn], q_rope[:nd], L.w_uk, L.w_uv_t, cache,
                                               fb.dec_block_tables, fb.dec_ctx_lens, c.softmax_scale)
        if T > nd:
            self._prefill_attention(L, torch.cat([q[nd:, :, :dn], q_rope[nd:]], -1), cache, fb, out[nd:])
        return out

    def _prefill_attention(self, L: _Layer, q: torch.Tensor, cache: torch.Tensor, fb, out: torch.Tensor):
        """Expanded MLA per prefill sequence: the context's latent rows through
        kv_b -> per-head K (nope | shared rope) and V; causal with the queries
        at the end of the context."""
        from .. import ops
        c = self.cfg
        nh, dn, dr, dv, r = c.num_attention_heads, c.qk_nope_head_dim, c.qk_rope_head_dim, c.v_head_dim, c.kv_lora_rank
        cu = fb.pre_cu_q.tolist()
        ctx = fb.pre_ctx_lens.tolist()
        for j, n in enumerate(ctx):
            a, b = cu[j], cu[j + 1]
            qn = b - a
            nblk = (n + BLOCK_SIZE - 1) // BLOCK_SIZE
            lat = cache[fb.pre_block_tables[j, :nblk].long()].reshape(-1, c.latent_dim)[:n]
            kvb = ops.linear(lat[:, :r].contiguous(), L.w_kvb).view(n, nh, dn + dv)
            k = torch.cat([kvb[..., :dn], lat[:, None, r:].expand(n, nh, dr)], -1)
            qpos = torch.arange(n - qn, n, device=q.device)
            mask = torch.arange(n, device=q.device)[None, :] <= qpos[:, None]
            o = F.scaled_dot_product_attention(q[a:b].transpose(0, 1), k.transpose(0, 1),
                                               kvb[..., dn:].transpose(0, 1), attn_mask=mask,
                                               scale=c.softmax_scale)
            out[a:b] = o.transpose(0, 1).reshape(qn, nh * dv)

    def _moe(self, M: _MoE, x: torch.Tensor, h: torch.Tensor, norm_w: torch.Tensor) -> torch.Tensor:
        """h += routed experts + shared expert; returns rmsnorm(h) * norm_w."""
        from .. import ops
        from .moe import routed_experts
        c = self.cfg
        idx, wts = route(c, x.float() @ M.router_w.t(), M.router_b)
        out = routed_experts(x, idx.to(torch.int32).contiguous(), wts.float().contiguous(), M.gu_w, M.gu_exp,
                             M.dn_w, M.dn_exp, c.n_routed_experts, c.moe_intermediate_size)
        if M.sh_gu is not None:
            ops.linear(ops.linear_swiglu(x, M.sh_gu), M.sh_dn, residual=h, out=h)
        return ops.rmsnorm(out, norm_w, c.rms_norm_eps, residual=h, residual_out=h)

    def forward_hidden(self, fb, kv: MLACache) -> torch.Tensor:
        from .. import ops
        c = self.cfg
        h = ops.embedding(fb.input_ids, self.embed)
        x = ops.rmsnorm(h, self.layers[0].ln1, c.rms_norm_eps)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            a = self._mla(i, L, x, fb, kv)
            ops.linear(a, L.wo, residual=h, out=h)
            x = ops.rmsnorm(h, L.ln2, c.rms_norm_eps)
            nw = self.layers[i + 1].ln1 if i + 1 < n else self.norm
            if L.moe is not None:
                x = self._moe(L.moe, x, h, nw)
            else:
                ops.linear(ops.linear_swiglu(x, L.w_gu), L.wd, residual=h, out=h)
                x = ops.rmsnorm(h, nw, c.rms_norm_eps)
        return x
