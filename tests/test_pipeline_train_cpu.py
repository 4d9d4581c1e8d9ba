"""Pipeline-parallel training (1F1B) on gloo ranks equals the single-process
trainer on the same global batch: losses, gradient norms and every parameter
after the optimizer steps (tied and untied embeddings, 2 and 3 stages)."""
import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rlx_models_b200 import config as C
from rlx_models_b200.train.trainer import TrainConfig, Trainer
from rlx_models_b200.weights.init import random_weights


def _cfg(tied):
    return C.tiny(num_hidden_layers=5, hidden_size=64, intermediate_size=128, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=16, vocab_size=96, tie_word_embeddings=tied)


def _batches(steps, B=6, S=10, V=96):
    return [torch.randint(0, V, (B, S + 1), generator=torch.Generator().manual_seed(s)) for s in range(steps)]


TC = dict(lr=1e-2, micro_batch=2, param_dtype="float32", grad_clip=0.5)


def _worker(rank, world, port, out_dir, steps, tied):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from rlx_models_b200.train.pipeline import PipelineTrainer
    cfg = _cfg(tied)
    t = PipelineTrainer(cfg, TrainConfig(**TC, activation_checkpointing=False), random_weights(cfg, 0),
                        stage=rank, stages=world, device="cpu")
    ms = [t.step(b) for b in _batches(steps)]
    torch.save({"losses": [m.loss for m in ms], "gnorms": [m.grad_norm for m in ms],
                "params": t.named_parameters()}, os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,tied", [(2, True), (3, False), (3, True)])
def test_pipeline_1f1b_matches_single_process(world, tied):
    steps = 3
    cfg = _cfg(tied)
    ref = Trainer(cfg, TrainConfig(**TC, activation_checkpointing=False), random_weights(cfg, 0), device="cpu")
    rm = [ref.step(b) for b in _batches(steps)]
    ref_params = {}
    for g in ref.model.groups:
        ref_params.update(g.named_full())
    with tempfile.TemporaryDirectory() as d:
        port = 29700 + (os.getpid() + world * 7 + tied) % 250
        mp.spawn(_worker, args=(world, port, d, steps, tied), nprocs=world, join=True)
        res = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    for r in range(world):
        for a, b in zip(res[r]["losses"], [m.loss for m in rm]):
            assert abs(a - b) < 1e-5 * max(1.0, abs(b))
        for a, b in zip(res[r]["gnorms"], [m.grad_norm for m in rm]):
            assert abs(a - b) < 1e-4 * max(1.0, abs(b))
    seen = set()
    for r in range(world):
        for n, t in res[r]["params"].items():
            key = "model.embed_tokens.weight" if (n == "lm_head.weight" and tied) else n
            assert torch.allclose(t, ref_params[key], rtol=1e-5, atol=1e-6), (r, n)
            seen.add(key)
    assert seen == set(ref_params)
