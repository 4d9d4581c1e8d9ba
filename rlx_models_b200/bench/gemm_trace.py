"""Per-CTA timeline of one tcgen05 GEMM launch (globaltimer stamps).

    python -m rlx_models_b200.bench.gemm_trace --M 64 --N 4096 --K 4096 [--splits 0] [--mode 0]

Stamps (ns, per CTA): 0 entry, 1 prologue done, 2 weight prefetch issued,
3 producer past griddepcontrol.wait, 4 first stage consumed by the MMA warp,
5 last MMA issued, 6 first accumulator ready in the epilogue, 7 split-K
arrival counted, 8 epilogue done, 9 exit. Prints medians / max relative to
the earliest entry, after flushing L2.
"""
from __future__ import annotations

import argparse

import torch

from .. import ops
from ..ops._ext import ext, scratch

NAMES = ["entry", "prologue", "prefetch", "pdl_wait", "first_stage", "last_mma", "acc_ready", "splitk_arrive",
         "epi_done", "exit"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--M", type=int, default=64)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--mode", type=int, default=0)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    x = torch.randn(args.M, args.K, device=dev).bfloat16()
    w = (torch.randn(args.N, args.K, device=dev) * 0.02).bfloat16()
    n_out = args.N // 2 if args.mode == 2 else args.N
    out = torch.empty(args.M, n_out, device=dev, dtype=torch.float32 if args.mode == 1 else torch.bfloat16)
    s = scratch(dev)
    trace = torch.zeros(148 * 16, dtype=torch.int64, device=dev)
    flush = torch.empty(256 << 18, dtype=torch.float32, device=dev)
    for it in range(3):
        flush.fill_(1.0)
        trace.zero_()
        torch.cuda.synchronize()
        ext().linear(x, w, out, args.mode, None, None, 1.0, s.gemm_ws, s.gemm_sem, s.status, -1, 0, args.splits,
                     trace)
        torch.cuda.synchronize()
    ops.check_errors(dev)
    t = trace.view(148, 16)[:, :10].cpu()
    used = t[:, 0] > 0
    t = t[used]
    t0 = t[:, 0].min()
    rel = (t - t0).float() / 1000.0
    rel[t == 0] = float("nan")
    print(f"CTAs: {int(used.sum())}  kernel span: {float(torch.nanquantile(rel[:, 9], 1.0)):.2f} us")
    for i, n in enumerate(NAMES):
        col = rel[:, i]
        col = col[~torch.isnan(col)]
        if col.numel():
            print(f"  {i} {n:14s} median {float(col.median()):8.2f} us   max {float(col.max()):8.2f} us  (n={col.numel()})")


if __name__ == "__main__":
    main()
