"""FLUX DiT sequence-parallel correctness check (launch with torchrun on N GPUs).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m rlx_models_b200.parallel.flux_sp_check

Runs one velocity evaluation of a small FLUX-shaped DiT (heads divisible by N)
split over N ranks (Ulysses all-to-all around the joint attention) and, on
rank 0, the same model on one GPU; the velocities must agree to bf16
tolerance, eagerly and through the CUDA graph. Prints one JSON line.
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
    from rlx_models_b200 import ops
    from rlx_models_b200.config import flux_tiny
    from rlx_models_b200.models.flux import FluxDiT
    from rlx_models_b200.models.flux_common import flux_random_weights

    heads = max(2, world)
    cfg = flux_tiny(hidden_size=128 * heads, num_heads=heads, mlp_ratio=2.0)
    w = flux_random_weights(cfg, seed=1, bias_std=0.02)
    B, Lt, h, wd = 2, 64, 8, 8
    g = torch.Generator().manual_seed(2)
    img = torch.randn(B, h * wd, cfg.in_channels, generator=g).to(dev).bfloat16()
    txt = torch.randn(B, Lt, cfg.context_in_dim, generator=g).to(dev).bfloat16()
    y = torch.randn(B, cfg.vec_in_dim, generator=g).to(dev).bfloat16()
    t, gd = torch.tensor([0.7, 0.2]), torch.tensor([3.5, 3.5])
    sp = FluxDiT(cfg, w, device=dev, sp_rank=rank, sp_size=world)
    v_eager = sp.forward(img, txt, t, y, gd, h, wd, graph=False).clone()
    v_graph = sp.forward(img, txt, t, y, gd, h, wd).clone()
    torch.cuda.synchronize(dev)
    ops.check_errors(dev)
    ok = torch.equal(v_eager, v_graph)
    res = {"world": world, "eager_equals_graph": ok}
    if rank == 0:
        ref = FluxDiT(cfg, w, device=dev).forward(img, txt, t, y, gd, h, wd, graph=False)
        rel = float((v_eager.float() - ref.float()).norm() / ref.float().norm())
        ok = ok and rel < 1e-2
        res.update(rel_err_vs_one_gpu=rel, ok=ok)
        print(json.dumps(res), flush=True)
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    sp._graph = None  # release the graph (it holds NCCL work) before tearing the group down
    torch.cuda.synchronize(dev)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(int(flag.item() != 0))


if __name__ == "__main__":
    main()
