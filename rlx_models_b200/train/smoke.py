"""One tiny training step on the GPU for the package smoke check: forward and
backward through the tcgen05 GEMMs and the fused lm_head + cross-entropy,
gradient push into the shard, fused AdamW."""
from __future__ import annotations

import torch


def train_smoke(dev: torch.device) -> None:
    from .. import config as C
    from .. import ops
    from ..weights.init import random_weights
    from .trainer import TrainConfig, Trainer
    cfg = C.tiny(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                 num_key_value_heads=2, head_dim=64, vocab_size=512)
    t = Trainer(cfg, TrainConfig(lr=1e-3, micro_batch=2), random_weights(cfg, 0), device=dev)
    batch = torch.randint(0, cfg.vocab_size, (4, 65), generator=torch.Generator().manual_seed(0))
    m0 = t.step(batch)
    m1 = t.step(batch)
    ops.check_errors(dev)
    assert torch.isfinite(torch.tensor([m0.loss, m1.loss])).all() and m1.loss < m0.loss, (m0.loss, m1.loss)
    if t.push is not None:
        t.push.close()
