"""One-GPU emulation of the peer-memory collective kernels, for profiling.

    python -m rlx_models_b200.parallel.collective_emu --op pull|pull2|argmax|combine [--world 8] [--M 64]

``ncu`` never runs a multi-rank command, so the fused collective kernels
(``ar_pull_norm``, ``ar2_norm``, ``tp_argmax``, ``ep_combine_norm``) are
captured here as ONE rank of a ``--world``-rank job on one GPU: every entry of
the peer tables points at a separate buffer in this GPU's memory (the same
number of bytes the real rank reads from its peers, but from local HBM / L2
instead of over NVLink), and every flag the kernel waits on is set before the
launch, so no launch waits for another (the flag stores meant for other ranks
go to a dummy array, the ones for this rank to its real flags; the argmax, whose keys carry their op's tag, gets the
other ranks' keys written before each launch, a small fill kernel that the
graph timing includes). What this measures is the kernel's own cost - its
loads, reduction, norm and stores - with the NVLink transfer and the
cross-rank skew taken out; the multi-rank timing (``comm_bench``) adds them
back. Each op runs ``--iters`` plain launches (ncu) and, with ``--time``,
CUDA-event timing of a graph of ``--reps`` launches.
"""
from __future__ import annotations

import argparse
import json

import torch

FLAG_SET = 0x7FFFFFFF  # above any epoch a run reaches: every bounded wait passes at once


def _ptrs(ts, dev):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=dev)


def build(op: str, world: int, M: int, H: int, dev, vocab: int = 151936, k: int = 4, experts: int = 128):
    """Buffers and a zero-argument launch for one rank (rank 0) of ``op``;
    returns (launch, peer_bytes, bufs): ``peer_bytes`` is what the real rank
    moves over NVLink per launch, ``bufs`` the named tensors (inputs and
    outputs, kept alive by the caller)."""
    from ..ops._ext import ext, scratch
    s = scratch(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    rank = 0
    # the other ranks' flags preset; this rank's own entries are raised by the kernel
    # itself (its flag stores to "rank 0" land in the real flag array), so a kernel
    # that waits on its own CTAs (the two-shot reduction's barrier 2) still orders them
    flags = torch.full((2 * world,), FLAG_SET, dtype=torch.int32, device=dev)
    flags[rank] = 0
    flags[world + rank] = 0
    dummy = torch.zeros(2 * world, dtype=torch.int32, device=dev)
    peer_flags = _ptrs([flags if q == rank else dummy for q in range(world)], dev)
    h = (torch.randn(M, H, device=dev, generator=g) * 0.1).bfloat16()
    nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
    out = torch.empty_like(h)
    keep = dict(flags=flags, dummy=dummy, peer_flags=peer_flags, h=h, nw=nw, out=out)
    if op in ("pull", "pull2"):
        rows = 128
        accs = [torch.randn(rows, H, device=dev, generator=g) * 0.01 for _ in range(world)]
        zero = torch.zeros(rows, H, device=dev)
        peer_acc = _ptrs(accs, dev)
        keep.update(accs=accs, zero=zero, peer_acc=peer_acc)
        if op == "pull":
            ctr = torch.zeros(2, dtype=torch.int32, device=dev)
            keep.update(ctr=ctr)

            def launch():
                ext().ar_pull_norm(peer_acc, peer_flags, flags, zero, rows, h, nw, out, ctr[0:1], ctr[1:2], rank,
                                   world, 1e-6, s.status)
            # fp32 partial rows of every other rank
            return launch, (world - 1) * M * H * 4, keep
        rpr_max = (rows + world - 1) // world
        rpr = (M + world - 1) // world
        # result slots: [rpr_max][H] bf16 residual rows, then fp32 slice sums of squares
        res = [torch.zeros(2, rpr_max, H, device=dev, dtype=torch.bfloat16) for _ in range(world)]
        peer_res = _ptrs(res, dev)
        ctr2 = torch.zeros(3, dtype=torch.int32, device=dev)
        keep.update(res=res, peer_res=peer_res, ctr=ctr2, rpr=rpr)

        def launch():
            ext().ar2_norm(peer_acc, peer_res, res[rank], peer_flags, flags, zero, rows, h, nw, out, ctr2[0:1],
                           ctr2[1:3], rank, world, rpr, rpr_max, 1e-6, s.status)
        # reduce-scatter reads (fp32, owned rows from every peer) + gather reads (bf16 residual rows
        # of the rows other ranks own, plus their slice sums of squares)
        return launch, (world - 1) * rpr * H * 4 + (world - 1) * rpr * (H * 2 + H // 512 * 4), keep
    if op == "argmax":
        R, Vl, max_rows = M, vocab // world, 256
        logits = torch.randn(R, Vl, device=dev, generator=g)
        keys = torch.zeros(2, max_rows, world, dtype=torch.int64, device=dev)
        peer_keys = _ptrs([keys] * world, dev)
        ctr = torch.zeros(2, dtype=torch.int32, device=dev)
        picked = torch.empty(R, dtype=torch.int32, device=dev)
        keep.update(logits=logits, keys=keys, peer_keys=peer_keys, ctr=ctr, picked=picked)

        def launch():
            # the other ranks' keys of this op: value bits 0 (lose to any real value) and this
            # op's tag, computed on the device from the epoch counter (so graph replays stay valid)
            e = ctr[0:1].long() + 1
            keys.index_copy_(0, e & 1, (1 + e % 8191).view(1, 1, 1).expand(1, max_rows, world).contiguous())
            ext().tp_argmax(logits, rank * Vl, keys, peer_keys, ctr[0:1], ctr[1:2], picked, max_rows, rank, world,
                            s.status)
        return launch, (world - 1) * R * 8, keep
    if op == "combine":
        T = M
        e_local = experts // world
        rows = [(torch.randn(T * k, H, device=dev, generator=g) * 0.05).bfloat16() for _ in range(world)]
        inv = [torch.arange(T * k, dtype=torch.int32, device=dev) for _ in range(world)]
        ex = torch.randint(0, experts, (T, k), generator=torch.Generator().manual_seed(1)).to(dev, torch.int32)
        ctr = torch.zeros(2, dtype=torch.int32, device=dev)
        peer_rows, peer_inv = _ptrs(rows, dev), _ptrs(inv, dev)
        keep.update(rows=rows, inv=inv, experts=ex, e_local=e_local, ctr=ctr, peer_rows=peer_rows,
                    peer_inv=peer_inv)

        def launch():
            ext().ep_combine_norm(peer_rows, peer_inv, peer_flags, flags, ex, e_local, h, nw, out, ctr[0:1],
                                  ctr[1:2], rank, world, 1e-6, s.status)
        remote = int((ex // e_local != rank).sum())  # expert rows owned by other ranks
        return launch, remote * H * 2, keep
    raise ValueError(f"unknown op {op!r}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="pull", choices=["pull", "pull2", "argmax", "combine"])
    ap.add_argument("--world", type=int, default=8)
    ap.add_argument("--M", type=int, default=64, help="rows (tokens) per launch")
    ap.add_argument("--H", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=3, help="plain launches (for an ncu capture)")
    ap.add_argument("--time", action="store_true", help="also CUDA-event time a graph of --reps launches")
    ap.add_argument("--reps", type=int, default=200)
    args = ap.parse_args()
    from .. import ops
    if not 1 <= args.world <= 8:
        raise SystemExit("--world must be 1..8")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    launch, peer_bytes, _keep = build(args.op, args.world, args.M, args.H, dev)
    for _ in range(args.iters):
        launch()
    torch.cuda.synchronize(dev)
    ops.check_errors(dev)
    res = {"op": args.op, "world": args.world, "M": args.M, "H": args.H, "peer_bytes": peer_bytes,
           "nvlink_floor_us": round(peer_bytes / 770e9 * 1e6, 2)}
    if args.time:
        gr = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            launch()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(gr):
            for _ in range(args.reps):
                launch()
        gr.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gr.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        ops.check_errors(dev)
        res["local_us_per_launch"] = round(e0.elapsed_time(e1) / args.reps * 1e3, 2)
        del gr
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
