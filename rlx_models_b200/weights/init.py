"""HF tensor-name contracts and seeded random initialisation.

Every tensor gets its own generator seeded from ``seed`` and the CRC32 of
its name, so any subset (a TP/EP/FSDP rank's shard, one layer) regenerates
bit-identically without materialising the rest. Matrices are N(0, std),
norm weights 1, biases 0 (HF ``_init_weights`` conventions); the reference's
synthetic-weight tests use the same "seeded, per-layer distinct" rule
(rlx-qwen3 src/synth.rs, src/lib.rs:140-245 synthetic name map).
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass

import torch

from ..config import DecoderConfig


@dataclass
class TensorSpec:
    name: str
    shape: tuple
    kind: str  # "matrix" | "norm" | "bias" | "mxfp4_blocks" | "mxfp4_scales" | "sinks"
    dtype: torch.dtype = torch.bfloat16


def decoder_tensor_specs(cfg: DecoderConfig) -> list[TensorSpec]:
    H, V, D = cfg.hidden_size, cfg.vocab_size, cfg.head_dim
    q, kv = cfg.q_size, cfg.kv_size
    specs = [TensorSpec("model.embed_tokens.weight", (V, H), "matrix")]
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        specs += [
            TensorSpec(p + "input_layernorm.weight", (H,), "norm"),
            TensorSpec(p + "post_attention_layernorm.weight", (H,), "norm"),
            TensorSpec(p + "self_attn.q_proj.weight", (q, H), "matrix"),
            TensorSpec(p + "self_attn.k_proj.weight", (kv, H), "matrix"),
            TensorSpec(p + "self_attn.v_proj.weight", (kv, H), "matrix"),
            TensorSpec(p + "self_attn.o_proj.weight", (H, q), "matrix"),
        ]
        if cfg.sandwich_norm:
            specs += [TensorSpec(p + "pre_feedforward_layernorm.weight", (H,), "norm"),
                      TensorSpec(p + "post_feedforward_layernorm.weight", (H,), "norm")]
        if cfg.qk_norm:  # per head (D), or over all heads of the token (MiniMax-M2)
            qn, kn = (q, kv) if cfg.qk_norm_full else (D, D)
            specs += [TensorSpec(p + "self_attn.q_norm.weight", (qn,), "norm"),
                      TensorSpec(p + "self_attn.k_norm.weight", (kn,), "norm")]
        if cfg.attention_bias:
            specs += [TensorSpec(p + "self_attn.q_proj.bias", (q,), "bias"),
                      TensorSpec(p + "self_attn.k_proj.bias", (kv,), "bias"),
                      TensorSpec(p + "self_attn.v_proj.bias", (kv,), "bias")]
            if cfg.model_type == "gpt_oss":
                specs.append(TensorSpec(p + "self_attn.o_proj.bias", (H,), "bias"))
        if cfg.attn_sinks:
            specs.append(TensorSpec(p + "self_attn.sinks", (cfg.num_attention_heads,), "sinks", torch.float32))
        if cfg.is_moe and cfg.model_type == "gpt_oss":
            E, I = cfg.num_experts, cfg.moe_intermediate_size
            specs += [TensorSpec(p + "mlp.router.weight", (E, H), "matrix"),
                      TensorSpec(p + "mlp.router.bias", (E,), "bias")]
            if cfg.expert_quant == "mxfp4":
                specs += [
                    TensorSpec(p + "mlp.experts.gate_up_proj_blocks", (E, 2 * I, H // 32, 16), "mxfp4_blocks",
                               torch.uint8),
                    TensorSpec(p + "mlp.experts.gate_up_proj_scales", (E, 2 * I, H // 32), "mxfp4_scales",
                               torch.uint8),
                    TensorSpec(p + "mlp.experts.down_proj_blocks", (E, H, I // 32, 16), "mxfp4_blocks", torch.uint8),
                    TensorSpec(p + "mlp.experts.down_proj_scales", (E, H, I // 32), "mxfp4_scales", torch.uint8),
                ]
            else:
                specs += [TensorSpec(p + "mlp.experts.gate_up_proj", (E, H, 2 * I), "matrix"),
                          TensorSpec(p + "mlp.experts.down_proj", (E, I, H), "matrix")]
            specs += [TensorSpec(p + "mlp.experts.gate_up_proj_bias", (E, 2 * I), "bias"),
                      TensorSpec(p + "mlp.experts.down_proj_bias", (E, H), "bias")]
        elif cfg.is_moe and cfg.is_moe_layer(i):
            E, I = cfg.num_experts, cfg.moe_intermediate_size
            specs.append(TensorSpec(p + "mlp.gate.weight", (E, H), "matrix"))
            if cfg.router_scoring == "sigmoid":
                specs.append(TensorSpec(p + "mlp.gate.e_score_correction_bias", (E,), "sinks", torch.float32))
            if cfg.n_shared_experts:
                Is = I * cfg.n_shared_experts
                ps = p + "mlp.shared_experts."
                specs += [TensorSpec(ps + "gate_proj.weight", (Is, H), "matrix"),
                          TensorSpec(ps + "up_proj.weight", (Is, H), "matrix"),
                          TensorSpec(ps + "down_proj.weight", (H, Is), "matrix")]
            for e in range(E):
                pe = p + f"mlp.experts.{e}."
                specs += [TensorSpec(pe + "gate_proj.weight", (I, H), "matrix"),
                          TensorSpec(pe + "up_proj.weight", (I, H), "matrix"),
                          TensorSpec(pe + "down_proj.weight", (H, I), "matrix")]
            Is = cfg.shared_expert_intermediate_size
            if Is:
                ps = p + "mlp.shared_expert."
                specs += [TensorSpec(ps + "gate_proj.weight", (Is, H), "matrix"),
                          TensorSpec(ps + "up_proj.weight", (Is, H), "matrix"),
                          TensorSpec(ps + "down_proj.weight", (H, Is), "matrix"),
                          TensorSpec(p + "mlp.shared_expert_gate.weight", (1, H), "matrix")]
        else:
            I = cfg.intermediate_size
            specs += [TensorSpec(p + "mlp.gate_proj.weight", (I, H), "matrix"),
                      TensorSpec(p + "mlp.up_proj.weight", (I, H), "matrix"),
                      TensorSpec(p + "mlp.down_proj.weight", (H, I), "matrix")]
    specs.append(TensorSpec("model.norm.weight", (H,), "norm"))
    if not cfg.tie_word_embeddings:
        specs.append(TensorSpec("lm_head.weight", (V, H), "matrix"))
    return specs


def tensor_seed(seed: int, name: str) -> int:
    return (int(seed) * 1_000_003 + zlib.crc32(name.encode())) & 0x7FFF_FFFF_FFFF


def init_tensor(spec: TensorSpec, seed: int, device="cpu", dtype: torch.dtype | None = None,
                std: float = 0.02) -> torch.Tensor:
    dt = dtype if (dtype is not None and spec.kind in ("matrix", "norm", "bias")) else spec.dtype
    dev = torch.device(device)
    if spec.kind == "norm":
        return torch.ones(spec.shape, dtype=dt, device=dev)
    if spec.kind == "bias":
        return torch.zeros(spec.shape, dtype=dt, device=dev)
    g = torch.Generator(device=dev).manual_seed(tensor_seed(seed, spec.name))
    if spec.kind == "sinks":
        return torch.randn(spec.shape, generator=g, device=dev, dtype=torch.float32) * std
    if spec.kind == "mxfp4_blocks":
        return torch.empty(spec.shape, dtype=torch.uint8, device=dev).random_(0, 256, generator=g)
    if spec.kind == "mxfp4_scales":
        # E8M0 exponents around 2^-8 give element magnitudes ~N(0, 0.02)-like
        return torch.randint(118, 121, spec.shape, generator=g, device=dev, dtype=torch.int64).to(torch.uint8)
    out = torch.empty(spec.shape, dtype=torch.float32 if dev.type == "cpu" else dt, device=dev)
    out.normal_(0.0, std, generator=g)
    return out.to(dt)


def random_weights(cfg: DecoderConfig, seed: int = 0, device="cpu", dtype: torch.dtype = torch.bfloat16,
                   names: set[str] | None = None) -> dict[str, torch.Tensor]:
    out = {}
    for spec in decoder_tensor_specs(cfg):
        if names is not None and spec.name not in names:
            continue
        out[spec.name] = init_tensor(spec, seed, device, dtype)
    return out
