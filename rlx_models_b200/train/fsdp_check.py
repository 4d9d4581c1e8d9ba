"""Multi-GPU FSDP check (launch with torchrun): gradient reduce-scatter by
NVLink push against the NCCL reduce-scatter.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m rlx_models_b200.train.fsdp_check

A seeded small Qwen3-structured decoder trains 3 steps on the same global
batch (each rank its 1/N of the rows) with ``grad_reduce="push"`` and with
``grad_reduce="nccl"``; losses, gradient norms and every rank's fp32 master
shard must agree to the bf16 rounding of the NCCL path's weight gradients. Prints one JSON line from
rank 0 and exits non-zero on a mismatch.
"""
from __future__ import annotations

import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    from .. import config as C
    from .. import ops
    from ..weights.init import random_weights
    from .trainer import TrainConfig, Trainer

    cfg = C.tiny(num_hidden_layers=3, hidden_size=512, intermediate_size=1024, num_attention_heads=8,
                 num_key_value_heads=4, head_dim=64, vocab_size=1000, tie_word_embeddings=True)
    w = random_weights(cfg, 0)
    B = 2 * world
    batch = torch.randint(0, cfg.vocab_size, (B, 257), generator=torch.Generator().manual_seed(0))
    mine = batch[rank * 2:(rank + 1) * 2]
    runs = {}
    for mode in ("push", "nccl"):
        t = Trainer(cfg, TrainConfig(lr=1e-3, micro_batch=1, grad_reduce=mode), w, rank=rank, world=world,
                    device=dev)
        ms = [t.step(mine) for _ in range(3)]
        ops.check_errors(dev)
        runs[mode] = ([m.loss for m in ms], [m.grad_norm for m in ms], [g.master.clone() for g in t.model.groups])
        if t.push is not None:
            t.push.close()
        del t
        torch.cuda.synchronize(dev)
        dist.barrier()
    (lp, gp, mp), (ln, gn, mn) = runs["push"], runs["nccl"]
    loss_rel = max(abs(a - b) / abs(b) for a, b in zip(lp, ln))
    gn_rel = max(abs(a - b) / abs(b) for a, b in zip(gp, gn))
    m_rel = max(((a - b).norm() / b.norm().clamp_min(1e-12)).item() for a, b in zip(mp, mn))
    # the push adds fp32 weight gradients; the NCCL path reduces the bf16-rounded
    # dW autograd hands it: agreement to bf16 rounding, not bit for bit
    ok = loss_rel < 2e-3 and gn_rel < 1e-2 and m_rel < 5e-2 and lp[-1] < lp[0]
    t = torch.tensor([1.0 if ok else 0.0], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(json.dumps({"world": world, "loss_push": lp, "loss_nccl": ln, "loss_rel": loss_rel,
                          "grad_norm_rel": gn_rel, "master_rel": m_rel, "ok_all_ranks": bool(t.item() == 1.0)}),
              flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if t.item() == 1.0 else 1


if __name__ == "__main__":
    sys.exit(main())
