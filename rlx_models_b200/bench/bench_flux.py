"""FLUX.1-dev-shaped DiT benchmark.

19 double + 38 single blocks, hidden 3072, 24 x 128 heads, MLP 12288, 3-axis
RoPE (16/56/56), random-init N(0, 0.02) bf16 weights. Inputs for a 1024x1024
image: latent 16x128x128 N(0, 1) packed 2x2 into 4096 image tokens, a text
stream of 512 x 4096 N(0, 1) embeddings and a 768-d N(0, 1) pooled vector;
batch 4, guidance 3.5, 28 shifted-schedule Euler steps.

One timed "step" is one denoising step of the batch (velocity evaluation +
Euler update); ``value`` is images/s = batch / (28 x step time). ``e2e`` runs
one full 28-step generation through ``generate_latents`` (the public call),
wall-clocked, including the noise / embedding uploads and the latent read-back.
"""
from __future__ import annotations

import json
import os
import time


def bench_flux(args) -> int:
    import torch

    from .. import ops
    from ..config import flux1_dev
    from ..models.flux import FluxDiT, generate_latents
    from ..models.flux_common import flux_random_weights, pack, schedule
    from ..utils.clocks import ClockSampler

    import torch.distributed as dist
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if ws > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=timedelta(seconds=600), device_id=dev)
    cfg = flux1_dev()
    B, Lt, res, steps, guidance = 4, 512, 1024, 28, 3.5
    # sequence parallel over the job's ranks (Ulysses); weights replicated
    model = FluxDiT(cfg, flux_random_weights(cfg, seed=0, device=dev), device=dev, sp_rank=rank, sp_size=ws)
    g = torch.Generator().manual_seed(0)
    lat = torch.randn(B, 16, res // 8, res // 8, generator=g)
    txt_h = torch.randn(B, Lt, cfg.context_in_dim, generator=g).bfloat16().pin_memory()
    pooled_h = torch.randn(B, cfg.vec_in_dim, generator=g).bfloat16().pin_memory()
    txt, pooled = txt_h.to(dev), pooled_h.to(dev)
    x = pack(lat).to(dev, torch.float32)
    Li = x.shape[1]
    hw = res // 16
    ts = schedule(steps, Li, shift=True)
    gvec = torch.full((B,), guidance)

    def denoise_step(i):
        nonlocal x
        v = model.forward(x.to(torch.bfloat16), txt, torch.full((B,), ts[i % steps]), pooled, gvec, hw, hw)
        x.add_(v.float(), alpha=ts[(i % steps) + 1] - ts[i % steps])

    for i in range(args.warmup):
        denoise_step(i)
    torch.cuda.synchronize(dev)
    ops.check_errors(dev)
    if ws > 1:
        dist.barrier()
    n0 = ops.launch_count()
    sampler = ClockSampler(dev.index)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        denoise_step(i)
    e1.record()
    torch.cuda.synchronize(dev)
    if ws > 1:
        dist.barrier()
    sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t)
    launches = ops.launch_count() - n0
    # end to end: one full generation through the public call
    if ws > 1:
        dist.barrier()
    t0 = time.perf_counter()
    out = generate_latents(model, txt_h.to(dev, non_blocking=True), pooled_h.to(dev, non_blocking=True),
                           height=res, width=res, steps=steps, guidance=guidance, seed=1).cpu()
    e2e_s = time.perf_counter() - t0
    if ws > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t)
    ops.check_errors(dev)
    assert torch.isfinite(out).all()
    flops_step = _flops(cfg, B, Lt, Li)
    res_d = {
        "metric": "FLUX.1-dev-shape images/s (batch 4, 1024x1024, 28 steps) (part of: Qwen3-8B-shape TP8 output "
                  "tok/s/box; p50 TTFT & TPOT; FSDP train tok/s)",
        "value": round(B / (steps * ms / 1e3), 4), "unit": "images/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: N(0,1) latents / text embeddings / pooled vector (seeded); random-init N(0,0.02) weights",
        "config": {"model": "FLUX.1-dev-shape DiT (19 double + 38 single, h3072, 24x128, MLP 12288)",
                   "global_batch": B, "seq_len": f"{Lt} txt + {Li} img",
                   "parallelism": f"sp{ws} (Ulysses all-to-all)" if ws > 1 else "single GPU",
                   "guidance": guidance, "denoise_steps": steps,
                   "l2": "inputs larger than L2: each step streams 24 GB of weights and ~2 GB of activations",
                   "step": "one denoising step of the batch"},
        "tflops_per_s": round(flops_step / (ms / 1e3) / 1e12, 1),
        "clocks": sampler.summary(),
        "e2e": {"value": round(B / e2e_s, 4), "unit": "images/s via generate_latents (wall clock, 28 steps)",
                "h2d_bytes_per_step": int((txt_h.numel() * 2 + pooled_h.numel() * 2 + lat.numel() * 4) / steps),
                "d2h_bytes_per_step": int(out.numel() * 4 / steps)},
        "gpu_launches": int(launches), "impl": "ours",
    }
    if rank == 0:
        print(json.dumps(res_d))
    if ws > 1:
        model._graph = None  # graphs holding NCCL work go before the process group
        torch.cuda.synchronize(dev)
        dist.barrier()
        dist.destroy_process_group()
    return 0


def _flops(cfg, B, Lt, Li):
    H, M = cfg.hidden_size, cfg.mlp_hidden
    L = Lt + Li
    per_tok_double = 2 * (3 * H * H + H * H + 2 * H * M)
    per_tok_single = 2 * (H * (3 * H + M) + (H + M) * H)
    attn = 4 * L * L * H  # QK^T and PV per batch element and block
    return B * (cfg.depth * (L * per_tok_double + attn) + cfg.depth_single_blocks * (L * per_tok_single + attn))
