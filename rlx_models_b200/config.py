"""HF ``config.json`` -> typed model configs.

Covers the keys the reference's config layer reads (rlx-models-core
src/config.rs:181 `legacy_rope_keys`, :231 `from_hf_json`; rlx-qwen3
src/config.rs:20-136; rlx-gpt-oss gpt_oss_ops.rs; rlx-flux1 src/config.rs:24-150):
transformers-5 ``rope_parameters`` are folded back into the legacy
``rope_theta`` / ``rope_scaling`` keys, a nested ``text_config`` (VLM wrappers)
is merged into the top level, and family defaults fill missing keys.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any


def legacy_rope_keys(cfg: dict) -> dict:
    """Map transformers-5 ``rope_parameters`` onto ``rope_theta`` / ``rope_scaling``."""
    cfg = dict(cfg)
    rp = cfg.get("rope_parameters")
    if isinstance(rp, dict):
        if "rope_theta" in rp and "rope_theta" not in cfg:
            cfg["rope_theta"] = rp["rope_theta"]
        if "partial_rotary_factor" in rp and "partial_rotary_factor" not in cfg:
            cfg["partial_rotary_factor"] = rp["partial_rotary_factor"]
        kind = rp.get("rope_type", rp.get("type", "default"))
        if kind not in (None, "default") and not cfg.get("rope_scaling"):
            cfg["rope_scaling"] = {k: v for k, v in rp.items() if k != "rope_theta"}
    return cfg


def merge_text_config(cfg: dict) -> dict:
    tc = cfg.get("text_config")
    if isinstance(tc, dict):
        merged = dict(cfg)
        for k, v in tc.items():
            merged.setdefault(k, v) if k in ("model_type",) else merged.__setitem__(k, v)
        return merged
    return cfg


@dataclass
class DecoderConfig:
    """Normalised decoder description shared by the dense and MoE families."""
    model_type: str = "qwen3"
    vocab_size: int = 151936
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    rope_scaling: dict | None = None
    partial_rotary_factor: float = 1.0  # RoPE on the first head_dim * factor dims (GLM-4: 0.5)
    # Granite scalars: h = embed * embedding_multiplier; h += residual_multiplier * sublayer;
    # attention scale = attention_multiplier (0: 1/sqrt(head_dim)); logits / logits_scaling
    embedding_multiplier: float = 1.0
    residual_multiplier: float = 1.0
    attention_multiplier: float = 0.0
    logits_scaling: float = 1.0
    # Gemma axes: GeGLU MLP, (1 + w) RMSNorm weights, sandwich norms (post-attention /
    # pre- and post-feedforward), attention and final logit softcapping, a separate
    # RoPE base for sliding-window layers
    mlp_act: str = "silu"  # "silu" | "gelu_tanh"
    causal: bool = True  # False: a bidirectional encoder trunk (EuroBERT)
    norm_unit_offset: bool = False
    sandwich_norm: bool = False
    attn_softcap: float = 0.0
    final_softcap: float = 0.0
    rope_local_theta: float = 0.0
    max_position_embeddings: int = 40960
    tie_word_embeddings: bool = False
    qk_norm: bool = True
    qk_norm_full: bool = False  # one RMSNorm over all heads' q (and k) values (OLMo-2, MiniMax-M2)
    attention_bias: bool = False
    mlp_bias: bool = False
    # sliding window: per-layer list of "full_attention" / "sliding_attention"
    sliding_window: int = 0
    layer_types: list[str] | None = None
    # learned attention sinks (gpt-oss)
    attn_sinks: bool = False
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    router_bias: bool = False
    expert_bias: bool = False
    swiglu_limit: float = 0.0   # clamped SwiGLU (gpt-oss: 7.0)
    swiglu_alpha: float = 1.702
    norm_topk_prob: bool = True
    shared_expert_intermediate_size: int = 0  # qwen2-moe: a dense SwiGLU expert every token uses, sigmoid-gated
    softmax_after_topk: bool = False  # gpt-oss: top-k on logits, softmax over the k
    # DeepSeek-style routing (glm4_moe): sigmoid scores + e_score_correction_bias for the
    # choice, group-limited top-k, routed scaling; always-on shared experts; dense first layers
    router_scoring: str = "softmax"  # "softmax" | "sigmoid"
    n_group: int = 1
    topk_group: int = 1
    routed_scaling_factor: float = 1.0
    n_shared_experts: int = 0
    first_k_dense_replace: int = 0
    moe_layers: list | None = None  # explicit MoE layer indices (Llama-4 interleaves dense / MoE)
    # Llama-4 axes: per-layer RoPE on / off (1 / 0; NoPE layers every 4th), RoPE on interleaved
    # pairs, weightless RMS norm of q and k after RoPE on the RoPE layers, chunked attention on
    # the RoPE layers, query temperature on the NoPE layers
    rope_layers: list | None = None
    rope_interleaved: bool = False
    qk_l2_norm: bool = False
    attention_chunk_size: int = 0
    attn_temperature_tuning: bool = False
    floor_scale: float = 8192.0
    attn_scale: float = 0.1
    expert_quant: str = "bf16"  # "bf16" | "mxfp4"
    torch_dtype: str = "bfloat16"
    extra: dict = field(default_factory=dict)

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def is_moe_layer(self, i: int) -> bool:
        if self.moe_layers is not None:
            return self.is_moe and i in self.moe_layers
        return self.is_moe and i >= self.first_k_dense_replace

    def uses_rope(self, i: int) -> bool:
        return self.rope_layers is None or bool(self.rope_layers[i])

    def layer_window(self, i: int) -> int:
        if self.layer_types is not None and self.sliding_window:
            return self.sliding_window if self.layer_types[i] == "sliding_attention" else 0
        return 0

    def num_params(self) -> int:
        H, I, V, L = self.hidden_size, self.intermediate_size, self.vocab_size, self.num_hidden_layers
        attn = H * (self.q_size + 2 * self.kv_size) + self.q_size * H
        if self.is_moe:
            mlp = self.num_experts * 3 * H * self.moe_intermediate_size + H * self.num_experts
        else:
            mlp = 3 * H * I
        emb = V * H * (1 if self.tie_word_embeddings else 2)
        return L * (attn + mlp + 2 * H) + emb + H

    @classmethod
    def from_hf_dict(cls, raw: dict) -> "DecoderConfig":
        d = legacy_rope_keys(merge_text_config(raw))
        mt = d.get("model_type", "qwen3")
        if mt in ("qwen3_vl", "qwen3_vl_text", "qwen3_vl_moe", "qwen3_vl_moe_text"):
            # Qwen3-VL's language model is Qwen3 (dense or MoE); for text its interleaved
            # multimodal RoPE (three equal position ids) is the plain 1-D RoPE
            mt = "qwen3_moe" if "moe" in mt else "qwen3"
            d = dict(d, model_type=mt)
            if d.get("num_experts") is None and d.get("num_local_experts") is not None:
                d["num_experts"] = d["num_local_experts"]  # the MoE config's serialised name
            if isinstance(d.get("rope_scaling"), dict) and d["rope_scaling"].get("rope_type", "default") == "default":
                d["rope_scaling"] = None
        kw: dict[str, Any] = {}
        fields = {f.name for f in dataclasses.fields(cls)}
        for k in fields:
            if k in d and k != "extra":
                kw[k] = d[k]
        kw["model_type"] = mt
        if "head_dim" not in d or d.get("head_dim") is None:
            kw["head_dim"] = d["hidden_size"] // d["num_attention_heads"]
        if "num_key_value_heads" not in d:
            kw["num_key_value_heads"] = d["num_attention_heads"]
        if mt in ("qwen3", "qwen3_moe"):
            kw.setdefault("qk_norm", True)
            if mt == "qwen3_moe":
                kw["num_experts"] = d.get("num_experts", 0)
                kw["moe_intermediate_size"] = d.get("moe_intermediate_size", 0)
        elif mt == "mixtral":
            kw["qk_norm"] = False
            kw.setdefault("rms_norm_eps", d.get("rms_norm_eps", 1e-5))
            kw["num_experts"] = d.get("num_local_experts", 8)
            kw["num_experts_per_tok"] = d.get("num_experts_per_tok", 2)
            kw["moe_intermediate_size"] = d.get("intermediate_size", 14336)
            kw["norm_topk_prob"] = True
        elif mt == "minimax_m2":  # full-width QK-norm, partial RoPE, sigmoid routing with a correction bias
            kw["qk_norm"] = kw["qk_norm_full"] = True
            kw["num_experts"] = d.get("num_local_experts", 256)
            kw["num_experts_per_tok"] = d.get("num_experts_per_tok", 8)
            kw["moe_intermediate_size"] = d.get("intermediate_size", 1536)
            kw["router_scoring"] = "sigmoid"
            kw["norm_topk_prob"] = True
            for k, dflt in (("n_group", 1), ("topk_group", 1), ("routed_scaling_factor", 1.0),
                            ("n_shared_experts", 0), ("first_k_dense_replace", 0)):
                kw[k] = dflt
            if d.get("rotary_dim") and not d.get("partial_rotary_factor"):
                kw["partial_rotary_factor"] = d["rotary_dim"] / kw.get("head_dim", d.get("head_dim", 128))
        elif mt in ("llama4_text", "llama4"):  # Llama-4 (text): iRoPE + top-1 sigmoid experts + shared expert
            kw["model_type"] = "llama4_text"
            kw["qk_norm"] = False
            kw["qk_l2_norm"] = bool(d.get("use_qk_norm", True))
            kw.setdefault("rms_norm_eps", d.get("rms_norm_eps", 1e-5))
            kw["num_experts"] = d.get("num_local_experts", 16)
            kw["num_experts_per_tok"] = d.get("num_experts_per_tok", 1)
            kw["moe_intermediate_size"] = d.get("intermediate_size", 8192)
            kw["intermediate_size"] = d.get("intermediate_size_mlp", d.get("intermediate_size", 8192))
            kw["router_scoring"] = "llama4"
            kw["n_shared_experts"] = 1
            n = d["num_hidden_layers"]
            step = int(d.get("interleave_moe_layer_step", 1))
            kw["moe_layers"] = list(d["moe_layers"]) if d.get("moe_layers") is not None else \
                list(range(step - 1, n, step))
            every = int(d.get("no_rope_layer_interval", 4))
            kw["rope_layers"] = list(d["no_rope_layers"]) if d.get("no_rope_layers") else \
                [int((i + 1) % every != 0) for i in range(n)]
            kw["rope_interleaved"] = True
            kw["attention_chunk_size"] = int(d.get("attention_chunk_size") or 0)
            kw["attn_temperature_tuning"] = bool(d.get("attn_temperature_tuning", True))
            kw["floor_scale"] = float(d.get("floor_scale", 8192))
            kw["attn_scale"] = float(d.get("attn_scale", 0.1))
        elif mt == "qwen2_moe":
            kw["qk_norm"] = False
            kw["attention_bias"] = True
            kw["num_experts"] = d.get("num_experts", 60)
            kw["moe_intermediate_size"] = d.get("moe_intermediate_size", 1408)
            kw["shared_expert_intermediate_size"] = d.get("shared_expert_intermediate_size", 0)
            kw["norm_topk_prob"] = bool(d.get("norm_topk_prob", False))
        elif mt in ("gemma", "gemma2", "gemma3_text", "gemma3"):
            kw["qk_norm"] = mt.startswith("gemma3")
            kw["norm_unit_offset"] = True
            kw["sandwich_norm"] = mt != "gemma"
            act = d.get("hidden_activation") or d.get("hidden_act") or "gelu_pytorch_tanh"
            kw["mlp_act"] = "gelu_tanh" if "gelu" in act else "silu"
            kw["embedding_multiplier"] = float(d["hidden_size"]) ** 0.5
            if d.get("query_pre_attn_scalar"):
                kw["attention_multiplier"] = float(d["query_pre_attn_scalar"]) ** -0.5
            kw["attn_softcap"] = float(d.get("attn_logit_softcapping") or 0.0)
            kw["final_softcap"] = float(d.get("final_logit_softcapping") or 0.0)
            kw["tie_word_embeddings"] = d.get("tie_word_embeddings", True)
            kw.setdefault("rms_norm_eps", d.get("rms_norm_eps", 1e-6))
            n = d["num_hidden_layers"]
            if mt != "gemma" and not d.get("layer_types"):
                period = 2 if mt == "gemma2" else int(d.get("sliding_window_pattern", 6))
                kw["layer_types"] = ["full_attention" if (i + 1) % period == 0 else "sliding_attention"
                                     for i in range(n)]
            if mt == "gemma":
                kw["sliding_window"] = 0
            if d.get("use_bidirectional_attention"):  # EmbeddingGemma: an encoder over the Gemma-3 trunk
                kw["causal"] = False
                # files keep the full window; attention spans |q - k| < window // 2 + 1
                kw["sliding_window"] = int(d.get("sliding_window") or 0) // 2 + 1
            rp = raw.get("rope_parameters") or (merge_text_config(raw).get("rope_parameters"))
            if isinstance(rp, dict) and "full_attention" in rp:  # per-layer-type RoPE (Gemma-3)
                full, local = rp["full_attention"], rp.get("sliding_attention", {})
                kw["rope_theta"] = float(full.get("rope_theta", 1e6))
                kind = full.get("rope_type", "default")
                kw["rope_scaling"] = None if kind == "default" else {k: v for k, v in full.items() if k != "rope_theta"}
                kw["rope_local_theta"] = float(local.get("rope_theta", 1e4))
            elif d.get("rope_local_base_freq"):
                kw["rope_local_theta"] = float(d["rope_local_base_freq"])
        elif mt == "eurobert":  # Llama-shaped bidirectional encoder
            kw["qk_norm"] = False
            kw["causal"] = False
            kw.setdefault("rms_norm_eps", d.get("rms_norm_eps", 1e-5))
        elif mt in ("granite", "phi3"):
            kw["qk_norm"] = False
            kw.setdefault("rms_norm_eps", d.get("rms_norm_eps", 1e-5))
            rs = kw.get("rope_scaling")
            if rs and rs.get("rope_type", rs.get("type")) in ("longrope", "su"):
                rs = dict(rs)
                rs.setdefault("original_max_position_embeddings", d.get("original_max_position_embeddings", 4096))
                kw["rope_scaling"] = rs
        elif mt in ("llama", "mistral", "qwen2"):
            kw["qk_norm"] = False
            kw.setdefault("rms_norm_eps", d.get("rms_norm_eps", 1e-5))
            if mt == "qwen2":
                kw["attention_bias"] = True
        elif mt == "glm4_moe":
            kw["qk_norm"] = bool(d.get("use_qk_norm", False))
            kw["attention_bias"] = bool(d.get("attention_bias", False))
            kw.setdefault("rms_norm_eps", d.get("rms_norm_eps", 1e-5))
            kw["num_experts"] = d.get("n_routed_experts", 128)
            kw["num_experts_per_tok"] = d.get("num_experts_per_tok", 8)
            kw["moe_intermediate_size"] = d.get("moe_intermediate_size", 1408)
            kw["router_scoring"] = "sigmoid"
            for k, dflt in (("n_group", 1), ("topk_group", 1), ("routed_scaling_factor", 1.0),
                            ("n_shared_experts", 1), ("first_k_dense_replace", 1)):
                kw[k] = d[k] if d.get(k) is not None else dflt
            kw["norm_topk_prob"] = bool(d.get("norm_topk_prob", True))
            kw.setdefault("partial_rotary_factor", 0.5)
        elif mt == "gpt_oss":
            kw["qk_norm"] = False
            kw["attention_bias"] = True
            kw["attn_sinks"] = True
            kw["num_experts"] = d.get("num_local_experts", d.get("num_experts", 128))
            kw["num_experts_per_tok"] = d.get("num_experts_per_tok", d.get("experts_per_token", 4))
            kw["moe_intermediate_size"] = d.get("intermediate_size", 2880)
            kw["router_bias"] = True
            kw["expert_bias"] = True
            kw["swiglu_limit"] = d.get("swiglu_limit", 7.0)
            kw["softmax_after_topk"] = True
            kw["sliding_window"] = d.get("sliding_window", 128)
            if "layer_types" not in d:
                kw["layer_types"] = ["sliding_attention" if i % 2 == 0 else "full_attention"
                                     for i in range(d["num_hidden_layers"])]
            q = d.get("quantization_config") or {}
            kw["expert_quant"] = "mxfp4" if q.get("quant_method") == "mxfp4" else d.get("expert_quant", "bf16")
        kw["extra"] = {k: v for k, v in d.items() if k not in fields}
        return cls(**kw)

    @classmethod
    def from_file(cls, path: str) -> "DecoderConfig":
        if os.path.isdir(path):
            path = os.path.join(path, "config.json")
        with open(path) as f:
            return cls.from_hf_dict(json.load(f))

    def to_hf_dict(self) -> dict:
        d = {k: v for k, v in dataclasses.asdict(self).items() if k != "extra"}
        d.update(self.extra)
        if self.model_type in ("gpt_oss", "mixtral", "minimax_m2"):
            d["num_local_experts"] = self.num_experts
            d["intermediate_size"] = self.moe_intermediate_size
        if self.model_type == "glm4_moe":
            d["n_routed_experts"] = self.num_experts
            d["use_qk_norm"] = self.qk_norm
        return d

    def save(self, path: str):
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, "config.json"), "w") as f:
            json.dump(self.to_hf_dict(), f, indent=2)


# ---------------------------------------------------------------------------
# Named shapes used by the benchmarks and tests (random-init weights)
# ---------------------------------------------------------------------------

def qwen3_0_6b() -> DecoderConfig:
    return DecoderConfig(model_type="qwen3", vocab_size=151936, hidden_size=1024, intermediate_size=3072,
                         num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                         rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=True)


def qwen3_1_7b() -> DecoderConfig:
    return DecoderConfig(model_type="qwen3", vocab_size=151936, hidden_size=2048, intermediate_size=6144,
                         num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                         rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=True)


def qwen3_8b() -> DecoderConfig:
    return DecoderConfig(model_type="qwen3", vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                         num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
                         rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=False)


def gpt_oss_120b() -> DecoderConfig:
    L = 36
    return DecoderConfig(model_type="gpt_oss", vocab_size=201088, hidden_size=2880, intermediate_size=2880,
                         num_hidden_layers=L, num_attention_heads=64, num_key_value_heads=8, head_dim=64,
                         rms_norm_eps=1e-5, rope_theta=150000.0,
                         rope_scaling={"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                                       "original_max_position_embeddings": 4096, "truncate": False},
                         max_position_embeddings=131072, tie_word_embeddings=False, qk_norm=False,
                         attention_bias=True, sliding_window=128,
                         layer_types=["sliding_attention" if i % 2 == 0 else "full_attention" for i in range(L)],
                         attn_sinks=True, num_experts=128, num_experts_per_tok=4, moe_intermediate_size=2880,
                         router_bias=True, expert_bias=True, swiglu_limit=7.0, softmax_after_topk=True,
                         expert_quant="mxfp4")


def deepseek_v2_lite():
    """DeepSeek-V2-Lite shape (15.7B total, 2.4B active): MLA without q
    compression, 64 routed experts (top-6, softmax) + 2 shared."""
    from .models.deepseek import DeepseekConfig
    return DeepseekConfig.from_dict(dict(
        model_type="deepseek_v2", vocab_size=102400, hidden_size=2048, intermediate_size=10944,
        moe_intermediate_size=1408, num_hidden_layers=27, num_attention_heads=16, n_shared_experts=2,
        n_routed_experts=64, num_experts_per_tok=6, routed_scaling_factor=1.0, kv_lora_rank=512, q_lora_rank=None,
        qk_rope_head_dim=64, v_head_dim=128, qk_nope_head_dim=128, n_group=1, topk_group=1, topk_method="greedy",
        scoring_func="softmax", norm_topk_prob=False, first_k_dense_replace=1, max_position_embeddings=163840,
        rope_theta=10000.0, rope_scaling={"rope_type": "yarn", "factor": 40.0, "original_max_position_embeddings": 4096,
                                          "beta_fast": 32, "beta_slow": 1, "mscale": 0.707, "mscale_all_dim": 0.707},
        bos_token_id=100000, eos_token_id=100001))


PRESETS = {
    "deepseek-v2-lite": deepseek_v2_lite,
    "qwen3-0.6b": qwen3_0_6b,
    "qwen3-1.7b": qwen3_1_7b,
    "qwen3-8b": qwen3_8b,
    "gpt-oss-120b": gpt_oss_120b,
}


def preset(name: str) -> DecoderConfig:
    key = name.lower().replace("_", "-")
    for k, fn in PRESETS.items():
        if key.endswith(k):
            return fn()
    raise KeyError(f"unknown preset {name!r}; known: {sorted(PRESETS)}")


def tiny(model_type: str = "qwen3", **over) -> DecoderConfig:
    """A small config with the same structure, for tests."""
    base = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                num_attention_heads=4, num_key_value_heads=2, head_dim=64, rms_norm_eps=1e-6, rope_theta=1e6)
    if model_type == "gpt_oss":
        cfg = gpt_oss_120b()
        base.update(num_experts=8, num_experts_per_tok=2, moe_intermediate_size=256, intermediate_size=256,
                    num_hidden_layers=2, sliding_window=16, layer_types=["sliding_attention", "full_attention"],
                    rope_scaling=dict(cfg.rope_scaling), expert_quant="mxfp4")
        base.update(over)
        return dataclasses.replace(cfg, **base)
    base.update(over)
    return DecoderConfig(model_type=model_type, **base)


# ---------------------------------------------------------------------------
# FLUX.1 rectified-flow DiT (BFL checkpoint layout: double_blocks.* /
# single_blocks.*), after rlx-flux1 src/config.rs:24-150
# ---------------------------------------------------------------------------

@dataclass
class FluxConfig:
    in_channels: int = 64          # 16 latent channels x 2x2 patch
    out_channels: int = 64
    vec_in_dim: int = 768          # CLIP pooled vector
    context_in_dim: int = 4096     # T5 token embeddings
    hidden_size: int = 3072
    mlp_ratio: float = 4.0
    num_heads: int = 24
    depth: int = 19                # double-stream blocks
    depth_single_blocks: int = 38
    axes_dim: tuple = (16, 56, 56)
    theta: float = 10000.0
    qkv_bias: bool = True
    guidance_embed: bool = True    # [dev]: distilled guidance input
    eps: float = 1e-6

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def mlp_hidden(self) -> int:
        return int(self.hidden_size * self.mlp_ratio)

    @classmethod
    def from_shapes(cls, shape_of) -> "FluxConfig":
        """Infer the config from checkpoint tensor shapes (``shape_of(name) -> tuple | None``)."""
        img_in = shape_of("img_in.weight")
        hidden, in_ch = img_in
        head_dim = shape_of("double_blocks.0.img_attn.norm.query_norm.scale")[0]

        def count(prefix):
            n = 0
            while shape_of(f"{prefix}.{n}.norm.key_norm.scale" if prefix == "single_blocks"
                           else f"{prefix}.{n}.img_attn.norm.key_norm.scale") is not None:
                n += 1
            return n

        return cls(in_channels=in_ch, out_channels=shape_of("final_layer.linear.weight")[0],
                   vec_in_dim=shape_of("vector_in.in_layer.weight")[1],
                   context_in_dim=shape_of("txt_in.weight")[1], hidden_size=hidden,
                   mlp_ratio=shape_of("double_blocks.0.img_mlp.0.weight")[0] / hidden,
                   num_heads=hidden // head_dim, depth=count("double_blocks"),
                   depth_single_blocks=count("single_blocks"),
                   guidance_embed=shape_of("guidance_in.in_layer.weight") is not None)


def flux1_dev() -> FluxConfig:
    return FluxConfig()


def flux1_schnell() -> FluxConfig:
    return FluxConfig(guidance_embed=False)


def flux_tiny(**over) -> FluxConfig:
    base = dict(in_channels=16, out_channels=16, vec_in_dim=32, context_in_dim=64, hidden_size=256,
                num_heads=2, depth=2, depth_single_blocks=2, axes_dim=(16, 56, 56))
    base.update(over)
    return FluxConfig(**base)
