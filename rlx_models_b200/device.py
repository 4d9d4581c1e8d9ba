"""Device capabilities and parallelism planning.

``devices()`` describes every visible GPU (name, SMs, memory, compute
capability, clocks and NVLink peers through NVML when available, peer access
through CUDA). ``plan_parallelism`` picks tensor / expert / pipeline degrees
for a decoder on ``n`` GPUs of ``mem_bytes`` each: weights plus the KV cache
of the requested context must fit with headroom; on one NVSwitch node every
GPU pair has full bandwidth, so dense models prefer tensor parallelism up to
the number of KV heads, MoE models put experts on every GPU (EP) with
attention replicated, and pipeline stages are added only when tensor
parallelism cannot split further. ``expert_bytes_per_rank`` is the MoE
weight footprint of one EP rank.

Reference: crates/rlx-models-core src/device_capabilities.rs (device lists,
LM device priority, MoE offload memory).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


def _nvml():
    try:
        import pynvml  # nvidia_ml_py
        pynvml.nvmlInit()
        return pynvml
    except Exception:
        return None


def devices(nvml=None) -> list[dict]:
    """Visible CUDA devices (empty without CUDA). ``nvml`` may be a fake with
    the pynvml function names, for tests."""
    out = []
    if not torch.cuda.is_available():
        return out
    nv = nvml if nvml is not None else _nvml()
    n = torch.cuda.device_count()
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        d = {"index": i, "name": p.name, "sms": p.multi_processor_count, "total_bytes": p.total_memory,
             "capability": f"{p.major}.{p.minor}",
             "peers": [j for j in range(n) if j != i and torch.cuda.can_device_access_peer(i, j)]}
        if nv is not None:
            try:
                h = nv.nvmlDeviceGetHandleByIndex(i)
                mem = nv.nvmlDeviceGetMemoryInfo(h)
                d["free_bytes"] = mem.free
                d["sm_clock_mhz"] = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                d["max_sm_clock_mhz"] = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
                links = 0
                for ln in range(18):
                    try:
                        links += int(nv.nvmlDeviceGetNvLinkState(h, ln) == 1)
                    except Exception:
                        break
                d["nvlinks_active"] = links
            except Exception:
                pass
        out.append(d)
    return out


def weight_bytes(cfg, dtype_bytes: float = 2.0, expert_bytes: float | None = None) -> dict:
    """Bytes of the dense part and of the experts of a decoder config."""
    H, V, L = cfg.hidden_size, cfg.vocab_size, cfg.num_hidden_layers
    attn = H * (cfg.q_size + 2 * cfg.kv_size) + cfg.q_size * H
    emb = V * H * (1 if cfg.tie_word_embeddings else 2)
    if cfg.is_moe:
        eb = expert_bytes if expert_bytes is not None else (4.25 / 8 if cfg.expert_quant == "mxfp4" else dtype_bytes)
        experts = L * cfg.num_experts * 3 * H * cfg.moe_intermediate_size * eb
        dense = (L * (attn + H * cfg.num_experts + 2 * H) + emb + H) * dtype_bytes
    else:
        experts = 0.0
        dense = (L * (attn + 3 * H * cfg.intermediate_size + 2 * H) + emb + H) * dtype_bytes
    return {"dense": dense, "experts": experts, "total": dense + experts}


def kv_bytes(cfg, tokens: int, dtype_bytes: float = 2.0) -> float:
    return 2.0 * cfg.num_hidden_layers * cfg.kv_size * tokens * dtype_bytes


def expert_bytes_per_rank(cfg, ep: int) -> float:
    return weight_bytes(cfg)["experts"] / ep


@dataclass
class ParallelPlan:
    tp: int
    ep: int
    pp: int
    bytes_per_gpu: float
    fits: bool
    reason: str


def plan_parallelism(cfg, n_gpus: int, mem_bytes: float = 180e9, context_tokens: int = 0,
                     headroom: float = 0.85) -> ParallelPlan:
    w = weight_bytes(cfg)
    kv = kv_bytes(cfg, context_tokens)
    budget = mem_bytes * headroom
    if cfg.is_moe:
        ep = max(d for d in range(1, n_gpus + 1) if n_gpus % d == 0 and cfg.num_experts % d == 0)
        per = w["dense"] + w["experts"] / ep + kv  # attention replicated, experts sliced
        pp = 1
        while per > budget and pp < cfg.num_hidden_layers:
            pp *= 2
            per = (w["dense"] + w["experts"] / ep + kv) / pp
        return ParallelPlan(1, ep, pp, per, per <= budget,
                            "experts split over every GPU, attention replicated" +
                            (f", {pp} pipeline stages for memory" if pp > 1 else ""))
    tp_max = max(d for d in range(1, n_gpus + 1)
                 if n_gpus % d == 0 and cfg.num_key_value_heads % d == 0 and cfg.num_attention_heads % d == 0)
    tp = 1
    per = w["total"] + kv
    while per > budget and tp < tp_max:
        tp *= 2
        per = (w["total"] + kv) / tp
    pp = 1
    while per > budget and tp * pp * 2 <= n_gpus:
        pp *= 2
        per = (w["total"] + kv) / (tp * pp)
    reason = "fits on one GPU" if tp == 1 and pp == 1 else f"tensor parallel over {tp}" + \
        (f" x {pp} pipeline stages" if pp > 1 else "")
    return ParallelPlan(tp, 1, pp, per, per <= budget, reason)
