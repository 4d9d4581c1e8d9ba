"""Model-type -> builder registry and lazy random weight source.

The reference keeps an LM runner registry keyed by architecture
(rlx-models-core src/lm_registry.rs:75-320 `LmBuildOptions`,
`build_lm_runner`; src/model_registry.rs:35-116; `classify_config`
src/standard_decoder.rs:13388). Here ``model_type`` from config.json selects a
builder; families register themselves with :func:`register`.
"""
from __future__ import annotations

from typing import Callable

import torch

from .config import DecoderConfig
from .weights.init import decoder_tensor_specs, init_tensor

_BUILDERS: dict[str, Callable] = {}


def register(*model_types: str):
    def deco(fn):
        for mt in model_types:
            _BUILDERS[mt] = fn
        return fn
    return deco


def registered() -> list[str]:
    return sorted(_BUILDERS)


class RandomWeights:
    """WeightMap-compatible source that generates each tensor on first take()."""

    def __init__(self, cfg: DecoderConfig, seed: int, device, dtype=torch.bfloat16):
        self.specs = {s.name: s for s in decoder_tensor_specs(cfg)}
        self.seed, self.device, self.dtype = seed, torch.device(device), dtype

    def __contains__(self, name):
        return name in self.specs

    def take(self, name, **kw):
        return init_tensor(self.specs[name], self.seed, self.device, self.dtype)

    def __getitem__(self, name):
        return self.take(name)

    def keys(self):
        return list(self.specs)


@register("qwen3", "llama", "mistral", "qwen2", "granite", "phi3")
def _dense(cfg, weights, device, tp_rank, tp_size, comm):
    from .models.decoder import DecoderLM
    return DecoderLM(cfg, weights, device=device, tp_rank=tp_rank, tp_size=tp_size, comm=comm)


@register("gpt_oss", "qwen3_moe", "mixtral", "qwen2_moe", "glm4_moe", "minimax_m2", "llama4_text")
def _moe(cfg, weights, device, tp_rank, tp_size, comm):
    from .models.moe import MoEDecoderLM
    return MoEDecoderLM(cfg, weights, device=device, ep_rank=tp_rank, ep_size=tp_size, comm=comm)


@register("deepseek_v3", "deepseek_v2", "kimi_k2", "glm4_moe_lite", "glm_moe_dsa")
def _deepseek(cfg, weights, device, tp_rank, tp_size, comm):
    from .models.deepseek import DeepseekLM
    if tp_size != 1:
        raise NotImplementedError("DeepSeek MLA models run on one GPU per replica")
    return DeepseekLM(cfg, weights, device=device)


@register("qwen3_5_text", "qwen3_5", "qwen3_5_moe_text", "qwen3_5_moe", "qwen3_next")
def _qwen35(cfg, weights, device, tp_rank, tp_size, comm):
    from .models.qwen35 import Qwen35LM
    if tp_size != 1:
        raise NotImplementedError("Qwen3.5 hybrid models run on one GPU per replica")
    return Qwen35LM(cfg, weights, device=device)


@register("mamba2", "bamba", "nemotron_h")
def _ssm(cfg, weights, device, tp_rank, tp_size, comm):
    from .models.mamba2 import SSMHybridLM
    if tp_size != 1:
        raise NotImplementedError("Mamba-2 models run on one GPU per replica")
    return SSMHybridLM(cfg, weights, device=device)


@register("mamba", "falcon_mamba", "jamba")
def _mamba1(cfg, weights, device, tp_rank, tp_size, comm):
    from .models.mamba1 import Mamba1LM
    if tp_size != 1:
        raise NotImplementedError("Mamba-1 models run on one GPU per replica")
    return Mamba1LM(cfg, weights, device=device)


@register("minimax")
def _minimax(cfg, weights, device, tp_rank, tp_size, comm):
    from .models.minimax import MiniMaxLM
    if tp_size != 1:
        raise NotImplementedError("MiniMax-Text-01 runs on one GPU per replica")
    return MiniMaxLM(cfg, weights, device=device)


@register("lfm2")
def _lfm2(cfg, weights, device, tp_rank, tp_size, comm):
    from .models.lfm2 import Lfm2LM
    if tp_size != 1:
        raise NotImplementedError("LFM2 runs on one GPU per replica")
    return Lfm2LM(cfg, weights, device=device)


def build_model(cfg: DecoderConfig, weights=None, *, device="cuda", tp_rank=0, tp_size=1, comm=None, seed=0):
    fn = _BUILDERS.get(cfg.model_type)
    if fn is None:
        raise KeyError(f"no builder for model_type={cfg.model_type!r}; registered: {registered()}")
    if weights is None and cfg.model_type in ("deepseek_v3", "deepseek_v2", "kimi_k2", "glm4_moe_lite", "glm_moe_dsa"):
        from .models.deepseek import random_weights
        weights = random_weights(cfg, seed, device)
    elif weights is None and cfg.model_type in ("qwen3_5_text", "qwen3_5", "qwen3_5_moe_text", "qwen3_5_moe",
                                                "qwen3_next"):
        from .models.qwen35 import random_weights
        weights = random_weights(cfg, seed, device)
    elif weights is None and cfg.model_type in ("mamba2", "bamba"):
        from .models.mamba2 import random_weights
        weights = random_weights(cfg, seed, device)
    elif weights is None and cfg.model_type in ("mamba", "falcon_mamba", "jamba"):
        from .models.mamba1 import random_weights
        weights = random_weights(cfg, seed, device)
    elif weights is None and cfg.model_type == "lfm2":
        from .models.lfm2 import random_weights
        weights = random_weights(cfg, seed, device)
    elif weights is None and cfg.model_type == "minimax":
        from .models.minimax import random_weights
        weights = random_weights(cfg, seed, device)
    elif weights is None:
        weights = RandomWeights(cfg, seed, device)
    with torch.no_grad():
        return fn(cfg, weights, device, tp_rank, tp_size, comm)
