"""Attention prefill microbenchmark at model shapes.

    python -m rlx_models_b200.bench.bench_attn [--json out.json]
    B200_ATTN_LEGACY=1 python -m rlx_models_b200.bench.bench_attn   # the mma.sync kernel

Shapes: FLUX.1 joint attention (batch 4, 4608 tokens, 24 heads x 128,
non-causal, query rows through the page table), Qwen3-8B prefill (8 prompts
of 2048, 32 q / 8 kv heads, causal), gpt-oss prefill (4 x 1024, 64 q / 8 kv
heads x 64 is D=64 and stays on the mma.sync kernel). Graph-replayed, L2
flushed between repetitions; TFLOP/s counts the executed (unmasked) half of
causal attention.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from .. import ops
from .bench_ops import Timer, peaks


def case(name, B, L, Hq, Hkv, D, causal, q_paged, dev):
    nb = B * L // 16
    q = (torch.randn(B * L, Hq, D, device=dev) * 0.5).bfloat16()
    k = (torch.randn(nb, Hkv, 16, D, device=dev) * 0.5).bfloat16()
    v = torch.randn(nb, Hkv, 16, D, device=dev).bfloat16()
    bt = torch.arange(nb, dtype=torch.int32, device=dev).view(B, L // 16)
    ctx = torch.full((B,), L, dtype=torch.int32, device=dev)
    cu = (torch.arange(B + 1, dtype=torch.int32) * L).to(dev)
    out = torch.empty_like(q)

    def fn():
        ops.prefill_attention(q, k, v, bt, ctx, cu, L, scale=1 / math.sqrt(D), causal=causal, q_paged=q_paged,
                              out=out)
    flops = 4.0 * B * Hq * L * L * D * (0.5 if causal else 1.0)
    return name, fn, flops


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--only", default=None, help="run one case (name prefix) --iters times without timing (for ncu)")
    ap.add_argument("--iters", type=int, default=2)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hbm, tf, src = peaks()
    timer = Timer(dev)
    kernel = "mma.sync (legacy)" if os.environ.get("B200_ATTN_LEGACY") == "1" else "tcgen05 FMHA"
    rows = []
    for name, fn, flops in [
        case("flux_joint_b4_l4608_h24", 4, 4608, 24, 24, 128, False, True, dev),
        case("qwen3_8b_prefill_b8_l2048_g4", 8, 2048, 32, 8, 128, True, False, dev),
        case("gpt_oss_prefill_b4_l1024_d64", 4, 1024, 64, 8, 64, True, False, dev),
    ]:
        if args.only:
            if not name.startswith(args.only):
                continue
            for _ in range(args.iters):
                fn()
            torch.cuda.synchronize()
            ops.check_errors(dev)
            print("ran", name)
            continue
        t = timer(fn, reps=args.reps)
        r = {"case": name, "kernel": kernel, "us": round(t * 1e6, 1), "tflops": round(flops / t / 1e12, 1),
             "frac_of_bf16_peak": round(flops / t / 1e12 / tf, 3)}
        rows.append(r)
        print(json.dumps(r), flush=True)
    ops.check_errors(dev)
    if args.json:
        json.dump({"peaks": {"bf16_TFLOPs": tf, "source": src}, "rows": rows}, open(args.json, "w"), indent=1)


if __name__ == "__main__":
    main()
