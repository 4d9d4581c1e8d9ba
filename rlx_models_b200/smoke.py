"""Tiny end-to-end check on cuda:0: prefill + decode of a small Qwen3 through
the engine (tcgen05 GEMMs, paged attention, norm/RoPE, sampling) and, when the
training stack is present, one forward + backward + optimizer step."""
from __future__ import annotations

import torch


def run_smoke() -> None:
    from . import config as C
    from . import ops
    from .models.decoder import DecoderLM
    from .runtime.engine import EngineConfig, LLMEngine, SamplingParams
    from .weights.init import random_weights

    assert torch.cuda.is_available(), "smoke() needs a CUDA device"
    dev = torch.device("cuda", 0)
    cfg = C.tiny(num_hidden_layers=2, hidden_size=512, intermediate_size=1024, num_attention_heads=8,
                 num_key_value_heads=2, head_dim=128, vocab_size=1024)
    w = random_weights(cfg, seed=0)
    model = DecoderLM(cfg, w, device=dev)
    eng = LLMEngine(model, EngineConfig(max_num_seqs=4, max_batched_tokens=256, max_model_len=256, num_blocks=32))
    out = eng.generate([[1, 2, 3, 4, 5, 6, 7], [9, 8, 7]], SamplingParams(max_new_tokens=4, ignore_eos=True))
    assert all(len(o.token_ids) == 4 for o in out)
    ops.check_errors(dev)
    try:
        from .train.smoke import train_smoke
    except ImportError:
        train_smoke = None
    if train_smoke is not None:
        train_smoke(dev)
    torch.cuda.synchronize(dev)
    print("smoke ok:", [o.token_ids for o in out])
