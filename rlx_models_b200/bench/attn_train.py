"""Training attention microbenchmark: this package's causal GQA forward (tcgen05,
saves the log-sum-exp) and flash-style backward against torch's SDPA.

    python -m rlx_models_b200.bench.attn_train [--B 2] [--S 4096] [--hq 16] [--hkv 8] [--reps 10]

Shape default: Qwen3-1.7B attention (16 Q / 8 KV heads, head_dim 128) at the
fine-tune sequence length 4096. Forward and backward are timed separately with
CUDA events after warm-up, inputs regenerated outside the timed region; causal
FLOPs count half of the S x S score matrix (forward 2 GEMMs, backward 5).
``--iters N`` instead launches forward + backward N times without timing (for
an ncu capture).
"""
from __future__ import annotations

import argparse
import json

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--B", type=int, default=2)
    ap.add_argument("--S", type=int, default=4096)
    ap.add_argument("--hq", type=int, default=16)
    ap.add_argument("--hkv", type=int, default=8)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--iters", type=int, default=0)
    ap.add_argument("--no-sdpa", action="store_true")
    args = ap.parse_args()
    from .. import ops
    from ..train.functional import AttentionFn
    from .bench_ops import peaks

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, S, Hq, Hkv, D = args.B, args.S, args.hq, args.hkv, 128
    g = torch.Generator(device=dev).manual_seed(0)

    def inputs():
        q = torch.randn(B, S, Hq, D, device=dev, generator=g).bfloat16().requires_grad_()
        k = torch.randn(B, S, Hkv, D, device=dev, generator=g).bfloat16().requires_grad_()
        v = torch.randn(B, S, Hkv, D, device=dev, generator=g).bfloat16().requires_grad_()
        do = torch.randn(B, S, Hq, D, device=dev, generator=g).bfloat16()
        return q, k, v, do

    def ours(q, k, v):
        return AttentionFn.apply(q, k, v)

    def sdpa(q, k, v):
        o = torch.nn.functional.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                                             v.transpose(1, 2), is_causal=True, enable_gqa=True)
        return o.transpose(1, 2)

    if args.iters:
        for _ in range(args.iters):
            q, k, v, do = inputs()
            ours(q, k, v).backward(do)
        torch.cuda.synchronize(dev)
        ops.check_errors(dev)
        print("launched", args.iters)
        return

    def time(fn):
        tf = tb = 0.0
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        for it in range(args.reps + 3):
            q, k, v, do = inputs()
            torch.cuda.synchronize(dev)
            ev[0].record()
            o = fn(q, k, v)
            ev[1].record()
            o.backward(do)
            ev[2].record()
            torch.cuda.synchronize(dev)
            if it >= 3:
                tf += ev[0].elapsed_time(ev[1])
                tb += ev[1].elapsed_time(ev[2])
        return tf / args.reps, tb / args.reps

    fl_fwd = 4.0 * B * Hq * S * S * D / 2
    fl_bwd = 2.5 * fl_fwd
    _, tf_peak, src = peaks()
    res = {"B": B, "S": S, "Hq": Hq, "Hkv": Hkv, "D": D, "peak_src": src}
    impls = [("ours", ours)] + ([] if args.no_sdpa else [("sdpa", sdpa)])
    for name, fn in impls:
        f_ms, b_ms = time(fn)
        res[name] = {"fwd_ms": round(f_ms, 3), "bwd_ms": round(b_ms, 3),
                     "fwd_tflops": round(fl_fwd / f_ms / 1e9, 1), "bwd_tflops": round(fl_bwd / b_ms / 1e9, 1),
                     "fwd_frac_of_measured": round(fl_fwd / f_ms / 1e9 / tf_peak, 3),
                     "bwd_frac_of_measured": round(fl_bwd / b_ms / 1e9 / tf_peak, 3)}
    ops.check_errors(dev)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
