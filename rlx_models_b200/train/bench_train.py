"""FSDP fine-tuning benchmark.

Qwen3-1.7B shape (28 layers, hidden 2048, 16q/8kv x 128, SwiGLU 6144, vocab
151936, tied embeddings), bf16 params/activations with fp32 master weights,
AdamW (lr 1e-4, betas 0.9/0.95, wd 0.1), sequence length 4096, global batch 64
sequences of uniform-random token ids (fresh every step), next-token CE.
FSDP over all ranks of the job; each rank takes 64 / world sequences per step,
in micro-batches. One "step" is one full optimizer step over the global batch.
"""
from __future__ import annotations

import json
import os
import time


def bench_train(args) -> int:
    import torch
    import torch.distributed as dist

    from .. import ops
    from ..config import qwen3_1_7b
    from ..registry import RandomWeights
    from ..utils.clocks import ClockSampler
    from .trainer import TrainConfig, Trainer

    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=timedelta(seconds=600), device_id=dev)
    cfg = qwen3_1_7b()
    seq = getattr(args, "seq_len", 4096)
    gbatch = getattr(args, "global_batch", 64)
    assert gbatch % ws == 0
    local_b = gbatch // ws
    tcfg = TrainConfig(lr=1e-4, betas=(0.9, 0.95), weight_decay=0.1, grad_clip=1.0,
                       micro_batch=getattr(args, "micro_batch", 4), total_steps=20,
                       activation_checkpointing=bool(getattr(args, "act_ckpt", 0)),
                       grad_reduce=getattr(args, "grad_reduce", "push"))
    trainer = Trainer(cfg, tcfg, RandomWeights(cfg, 0, dev), rank=rank, world=ws, device=dev)
    g = torch.Generator().manual_seed(1234 + rank)
    host = torch.empty(local_b, seq + 1, dtype=torch.int64).pin_memory()

    def batch():
        host.copy_(torch.randint(0, cfg.vocab_size, (local_b, seq + 1), generator=g))
        return host

    for _ in range(args.warmup):
        trainer.step(batch())
    ops.check_errors(dev)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    n0 = ops.launch_count()
    sampler = ClockSampler(local)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    metrics = [trainer.step(batch()) for _ in range(args.steps)]
    e1.record()
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t0
    if ws > 1:
        dist.barrier()
    sampler.stop()
    ms = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([ms, wall], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, wall = float(t[0]), float(t[1])
    tokens = gbatch * seq * args.steps
    res = {
        "metric": "Qwen3-1.7B-shape FSDP train tok/s (part of: Qwen3-8B-shape TP8 output tok/s/box; p50 TTFT & "
                  "TPOT; FSDP train tok/s)",
        "value": round(tokens / (ms / 1e3), 1), "unit": "train tok/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16 (fp32 master)",
        "data": "synthetic uniform-random token ids, fresh per step; random-init weights",
        "config": {"model": "Qwen3-1.7B-shape", "global_batch": gbatch, "seq_len": seq,
                   "parallelism": f"fsdp{ws}", "micro_batch_per_rank": tcfg.micro_batch,
                   "activation_checkpointing": tcfg.activation_checkpointing, "grad_reduce": tcfg.grad_reduce,
                   "l2": "inputs larger than L2 (every micro-step streams >1 GB of activations)"},
        "loss_first": metrics[0].loss, "loss_last": metrics[-1].loss,
        "clocks": sampler.summary(),
        "e2e": {"value": round(tokens / wall, 1), "unit": "train tok/s via Trainer.step (wall clock)",
                "h2d_bytes_per_step": local_b * (seq + 1) * 8, "d2h_bytes_per_step": 8},
        "gpu_launches": int(ops.launch_count() - n0), "impl": "ours",
    }
    if rank == 0:
        print(json.dumps(res))
    if ws > 1:
        dist.destroy_process_group()
    return 0
