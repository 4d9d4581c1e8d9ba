"""Row-parallel op microbenchmark (launch with torchrun on N GPUs).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m rlx_models_b200.parallel.comm_bench [--M 64]

Times, per rank with CUDA events (max over ranks), the decoder's row-parallel
step ``h += allreduce(x @ w_shard.T); x_next = rmsnorm(h)`` at the Qwen3-8B
o_proj shape (K = 4096 / N) through each communicator, plus a bare NCCL
all-reduce of the same partial. Reports us/op and, for the fused path, the
fraction of its roofline max(GEMM at peak, HBM weight stream, NVLink bytes at
the measured 770 GB/s per direction).
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist


def _graph_us(fn, iters, dev):
    """Device time per call of ``fn`` replayed ``iters`` times in one CUDA graph (max over ranks)."""
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / iters * 1e3], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del g
    return round(float(t), 2)


def kernel_breakdown(args, rank, world, dev, x, w, nw, M, H):
    """Decode row-parallel op split into its kernels, each graph-timed alone:
    the local accumulate GEMM, the one-shot and two-shot reduction kernels
    (their accumulator already filled), and a bare cross-rank flag barrier."""
    from .. import ops
    from ..ops._ext import ext, scratch
    from .pull_tp import PullTPComm
    out = {}
    comm = PullTPComm(rank, world, dev, 1e-6, hidden=H, two_shot="off")
    h = torch.zeros(M, H, device=dev, dtype=torch.bfloat16)
    o = torch.empty_like(h)
    s = scratch(dev)
    out["gemm_acc"] = _graph_us(lambda: ops.linear_acc(x, w, acc=comm.acc[0, :M]), args.iters, dev)

    def pull():
        ext().ar_pull_norm(comm.peer_acc[0], comm.peer_flags, comm.flags, comm.acc[1], comm.ROWS, h, nw, o,
                           comm.ctr[0:1], comm.ctr[1:2], rank, world, 1e-6, s.status)

    def two_shot():
        rpr = (M + world - 1) // world
        ext().ar2_norm(comm.peer_acc[0], comm.peer_res, comm.res, comm.peer_flags2, comm.flags2, comm.acc[1],
                       comm.ROWS, h, nw, o, comm.ctr2[0:1], comm.ctr2[1:3], rank, world, rpr, comm.rpr_max, 1e-6,
                       s.status)

    out["ar_pull_norm"] = _graph_us(pull, args.iters, dev)
    out["ar2_norm"] = _graph_us(two_shot, args.iters, dev)
    from ..train.fsdp import FlatGroup, GradPush
    fg = FlatGroup("b", [("t", torch.zeros(1024))], rank, world, dev)
    gp = GradPush([fg], rank, world, dev)
    out["flag_barrier"] = _graph_us(gp.barrier, args.iters, dev)
    logits = torch.randn(64, 151936 // world, device=dev)
    picked = torch.empty(64, dtype=torch.int32, device=dev)
    out["greedy_argmax_v19k_r64"] = _graph_us(lambda: comm.argmax(logits, picked), args.iters, dev)
    ops.check_errors(dev)
    torch.cuda.synchronize(dev)
    dist.barrier()
    gp.close()
    comm.close()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=64)
    ap.add_argument("--H", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--graph", type=int, default=1)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    from .. import ops
    from .tp import make_tp_comm

    M, H, K = args.M, args.H, args.K // world
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(M, K, device=dev, generator=g).bfloat16()
    w = (torch.randn(H, K, device=dev, generator=g) * 0.02).bfloat16()
    nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
    res = {}
    variants = [("nccl", "nccl", {}), ("fused", "fused", {})]
    if M <= 128:  # the pull communicator's decode path, one-shot and two-shot
        variants += [("pull", "pull", {"two_shot": "off"}), ("pull2", "pull", {"two_shot": "on"})]
    for label, kind, kw in variants:
        comm = make_tp_comm(kind, rank, world, dev, 1e-6, max_tokens=max(M, 128), hidden=H, **kw)
        ids = torch.zeros(M, dtype=torch.int32, device=dev)
        table = torch.randn(8, H, device=dev).bfloat16()
        h = comm.embed(ids, table)
        comm.norm_in(h, nw)

        def op():
            comm.rowpar_add_norm(x, w, h, nw)

        for _ in range(5):
            op()
        torch.cuda.synchronize(dev)
        dist.barrier()
        fn = op
        if args.graph:
            gr = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                op()
            torch.cuda.current_stream(dev).wait_stream(s)
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(gr):
                for _ in range(args.iters):
                    op()
            fn = gr.replay
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if args.graph:
            fn()
        else:
            for _ in range(args.iters):
                fn()
        e1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / args.iters * 1e3], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[label] = round(float(t), 2)
        ops.check_errors(dev)
        if args.graph:
            del gr
        torch.cuda.synchronize(dev)
        dist.barrier()
        if hasattr(comm, "close"):
            comm.close()
    if M <= 128:
        res["pull_kernels_us"] = kernel_breakdown(args, rank, world, dev, x, w, nw, M, H)
    # per-kernel breakdown of the fused op (eager, events between launches)
    from ..ops._ext import ext, scratch
    comm = make_tp_comm("fused", rank, world, dev, 1e-6, max_tokens=max(M, 128), hidden=H)
    h = comm.embed(torch.zeros(M, dtype=torch.int32, device=dev), torch.randn(8, H, device=dev).bfloat16())
    comm.norm_in(h, nw)
    sc = scratch(dev)
    acc_mode = M <= 128
    comm.one_shot = False  # breakdown of the two-shot kernels
    comm.rpr = (M + world - 1) // world
    h = torch.zeros(comm.rpr, H, device=dev, dtype=torch.bfloat16)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    tg = tn = 0.0
    for it in range(args.iters + 5):
        dist.barrier()
        ev[0].record()
        if acc_mode:
            ext().linear_push(x, w, None, 3, False, comm.rpr, H, 0, rank, world, comm.peer_racc, comm.peer_rs,
                              comm.ctr[0:1], comm.ctr[2:3], sc.gemm_ws, sc.gemm_sem, sc.status)
        else:
            ext().linear_push(x, w, None, 0, False, comm.rpr, H, comm.slot_elems, rank, world, comm.peer_recv, comm.peer_rs,
                              comm.ctr[0:1], comm.ctr[2:3], sc.gemm_ws, sc.gemm_sem, sc.status)
        ev[1].record()
        comm._rs_norm_ag(None if acc_mode else comm.recv, h, nw, racc=comm.racc if acc_mode else None)
        ev[2].record()
        torch.cuda.synchronize(dev)
        if it >= 5:
            tg += ev[0].elapsed_time(ev[1])
            tn += ev[1].elapsed_time(ev[2])
    t = torch.tensor([tg / args.iters * 1e3, tn / args.iters * 1e3], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    res["fused_breakdown_us"] = {"gemm_push": round(float(t[0]), 2), "rs_norm_ag": round(float(t[1]), 2)}
    # the same GEMM without the push (local output) for comparison
    tl = 0.0
    for it in range(args.iters + 5):
        ev[0].record()
        if acc_mode:
            ops.linear_acc(x, w).zero_()
        else:
            ops.linear(x, w)
        ev[1].record()
        torch.cuda.synchronize(dev)
        if it >= 5:
            tl += ev[0].elapsed_time(ev[1])
    res["local_gemm_us"] = round(tl / args.iters * 1e3, 2)
    ops.check_errors(dev)
    comm.close()
    part = torch.randn(M, H, device=dev, dtype=torch.float32)
    for _ in range(5):
        dist.all_reduce(part)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.iters):
        dist.all_reduce(part)
    e1.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / args.iters * 1e3], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    res["nccl_allreduce_only_f32"] = round(float(t), 2)
    # roofline of one row-parallel op on this rank
    flops = 2.0 * M * H * K
    w_bytes = 2.0 * H * K
    link = 2.0 * (world - 1) / world * M * H * 2  # reduce-scatter + all-gather, bf16
    roof_us = max(flops / 1.6186e15, w_bytes / 6.449e12, link / 770e9) * 1e6
    res.update(world=world, M=M, H=H, K_per_rank=K, roofline_us=round(roof_us, 2),
               fused_frac_of_roofline=round(roof_us / res["fused"], 3))
    if rank == 0:
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
