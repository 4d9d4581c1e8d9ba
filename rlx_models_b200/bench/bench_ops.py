"""Per-op microbenchmarks at model shapes, with roofline fractions.

    python -m rlx_models_b200.bench.bench_ops [--model qwen3-8b] [--tp 1] [--json out.json]

For every GEMM of the decoder layer (decode M=64 and prefill M=8192) and the
decode / prefill attention, times this package's kernel and the cuBLAS
baseline (torch.matmul) with CUDA events after warm-up, flushing L2 (writing a
256 MB buffer) before every timed repetition, and reports achieved TB/s and
TFLOP/s against MEASURED_PEAKS.json (or the fallback 6.65 TB/s, 1.59 PF/s).
This is also the quantized/dense matmul bench (the reference's
bench_matmul_rlx role).
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from .. import ops
from ..config import preset


def peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return d["hbm_gbs"] / 1e3, d["bf16_tflops"], "measured"
    except Exception:
        return 6.65, 1590.0, "fallback"


class Timer:
    """Device time of ``fn`` with L2 flushed before every repetition.

    ``reps`` x (flush, fn) and ``reps`` x (flush) are each captured in a CUDA
    graph; t(fn) = (T(flush+fn) - T(flush)) / reps, so host launch overhead
    (absent in the graph-replayed engine) does not enter the number.
    """

    def __init__(self, dev, flush_mb=256):
        self.flush = torch.empty(flush_mb * (1 << 20) // 4, dtype=torch.float32, device=dev)

    def _graph(self, fn, reps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                self.flush.fill_(1.0)
                if fn is not None:
                    fn()
        return g

    @staticmethod
    def _time(g, n=3):
        best = float("inf")
        for _ in range(n):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            best = min(best, a.elapsed_time(b))
        return best * 1e-3

    def __call__(self, fn, reps=10, warmup=3):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        g1 = self._graph(fn, reps)
        g0 = self._graph(None, reps)
        return max(0.0, self._time(g1) - self._time(g0)) / reps


def gemm_rows(cfg, tp, M):
    H, I, q, kv, V = cfg.hidden_size, cfg.intermediate_size, cfg.q_size, cfg.kv_size, cfg.vocab_size
    return [("qkv", M, (q + 2 * kv) // tp, H, 0), ("o_proj+res", M, H, q // tp, 1),
            ("gate_up+swiglu", M, 2 * I // tp, H, 2), ("down+res", M, H, I // tp, 1),
            ("lm_head(f32)", min(M, 64), V // tp, H, 3)]


def wgrad(args, dev, timer, tf, hbm):
    """FSDP weight gradient at the Qwen3-1.7B gate|up shape (dW [12288, 2048]
    from T tokens): the dense fp32 GEMM, the same GEMM adding dW into a
    gradient shard through the push epilogue (world 1, 8 emulated shards on
    this GPU), and cuBLAS (bf16 out) for reference."""
    T, N, K = args.M, 12288, 2048
    dy = (torch.randn(T, N, device=dev) * 0.02).bfloat16()
    x = torch.randn(T, K, device=dev).bfloat16()
    W = 8
    shard_n = (N * K + W - 1) // W
    shard_n = (shard_n + 127) // 128 * 128
    shards = torch.zeros(W, shard_n, dtype=torch.float32, device=dev)
    table = torch.tensor([shards[i].data_ptr() for i in range(W)], dtype=torch.int64, device=dev)
    s = ops.scratch(dev)
    dw = torch.empty(N, K, dtype=torch.float32, device=dev)

    def push():
        ops.ext().gemm_push_shards(dy.t(), x, table, 0, shard_n, 1.0, s.gemm_ws, s.gemm_sem, s.status)

    if args.only == "wgrad_push":
        for _ in range(args.iters):
            push()
        torch.cuda.synchronize()
        ops.check_errors(dev)
        print("ran wgrad_push", T, N, K)
        return
    flops = 2.0 * T * N * K
    for name, fn in (("wgrad_dense_f32", lambda: ops.matmul(dy.t(), x, out=dw)), ("wgrad_push_shards", push),
                     ("wgrad_cublas_bf16", lambda: torch.matmul(dy.t(), x))):
        t = timer(fn, args.reps)
        row = dict(op=name, T=T, N=N, K=K, us=round(t * 1e6, 1), tflops=round(flops / t / 1e12, 1),
                   frac_flops=round(flops / t / 1e12 / tf, 3))
        print(json.dumps(row), flush=True)
    ops.check_errors(dev)


def decode_attn_rows(args, cfg, dev, timer, hbm, rows, write=True):
    """Decode attention over bf16 and float8 e4m3 pages (batch 64 at 1400 and
    2300 tokens of context; the pages spread over a cache larger than L2)."""
    Hq, Hkv, D = cfg.num_attention_heads // args.tp, cfg.num_key_value_heads // args.tp, cfg.head_dim
    for dt, esize, splits in ((torch.bfloat16, 2, 0), (torch.float8_e4m3fn, 1, 0), (torch.float8_e4m3fn, 1, 2),
                              (torch.float8_e4m3fn, 1, 3)):
        if splits and args.only != "decode_attn":
            continue
        for (B, ctx) in ((64, 1400), (64, 2300)):
            nbps = (ctx + 15) // 16
            NB = B * nbps + 1
            kc = torch.randn(NB, Hkv, 16, D, device=dev).to(dt)
            vc = torch.randn(NB, Hkv, 16, D, device=dev).to(dt)
            tables = torch.randperm(NB - 1, device=dev)[:B * nbps].view(B, nbps).int()
            ctxs = torch.full((B,), ctx, dtype=torch.int32, device=dev)
            q = torch.randn(B, Hq, D, device=dev).bfloat16()
            out = torch.empty_like(q)
            t = timer(lambda: ops.decode_attention(q, kc, vc, tables, ctxs, scale=1 / math.sqrt(D), out=out,
                                                   splits=splits), args.reps)
            byts = 2.0 * B * ctx * Hkv * D * esize
            rows.append(dict(op="decode_attn" if esize == 2 else "decode_attn_fp8", B=B, ctx=ctx, splits=splits,
                             us=round(t * 1e6, 1), tbs=round(byts / t / 1e12, 2),
                             frac_hbm=round(byts / t / 1e12 / hbm, 3)))
            print(json.dumps(rows[-1]), flush=True)
    if write and args.json:
        json.dump({"peaks": {"hbm_tbs": hbm}, "rows": rows}, open(args.json, "w"), indent=1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--json", default=None)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--only", default=None, help="run a single GEMM op (e.g. o_proj+res) at --M; 'wgrad' times "
                    "the FSDP weight-gradient GEMM (dense / shard push / cuBLAS) with --M tokens, "
                    "'wgrad_push' only launches the push GEMM --iters times (for ncu)")
    ap.add_argument("--M", type=int, default=64)
    ap.add_argument("--iters", type=int, default=3, help="with --only: plain launches (for ncu)")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = preset(args.model)
    hbm, tf, src = peaks()
    timer = Timer(dev)
    rows = []
    if args.only in ("wgrad", "wgrad_push"):
        return wgrad(args, dev, timer, tf, hbm)
    if args.only == "decode_attn":
        return decode_attn_rows(args, cfg, dev, timer, hbm, rows)
    if args.only:
        for name, m, n, k, mode in gemm_rows(cfg, args.tp, args.M):
            if name != args.only:
                continue
            x = torch.randn(m, k, device=dev).bfloat16()
            w = (torch.randn(n, k, device=dev) * 0.02).bfloat16()
            r = torch.randn(m, n, device=dev).bfloat16() if mode == 1 else None
            for _ in range(args.iters):
                if mode == 2:
                    ops.linear_swiglu(x, w)
                else:
                    ops.linear(x, w, residual=r, out_dtype=torch.float32 if mode == 3 else torch.bfloat16)
            torch.cuda.synchronize()
            ops.check_errors(dev)
            print("ran", name, m, n, k)
        return
    for M in (64, 8192):
        for name, m, n, k, mode in gemm_rows(cfg, args.tp, M):
            x = torch.randn(m, k, device=dev).bfloat16()
            w = (torch.randn(n, k, device=dev) * 0.02).bfloat16()
            r = torch.randn(m, n, device=dev).bfloat16() if mode == 1 else None
            if mode == 2:
                out = torch.empty(m, n // 2, device=dev, dtype=torch.bfloat16)
                f = lambda: ops.linear_swiglu(x, w, out=out)
            elif mode == 3:
                out = torch.empty(m, n, device=dev, dtype=torch.float32)
                f = lambda: ops.linear(x, w, out=out)
            else:
                out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
                f = lambda: ops.linear(x, w, out=out, residual=r)
            t = timer(f, args.reps)
            tc = timer(lambda: torch.matmul(x, w.t()), args.reps)
            flops = 2.0 * m * n * k
            byts = 2.0 * (m * k + n * k + m * n * (2 if mode == 1 else 1))
            rows.append(dict(op=name, M=m, N=n, K=k, us=round(t * 1e6, 1), cublas_us=round(tc * 1e6, 1),
                             tflops=round(flops / t / 1e12, 1), tbs=round(byts / t / 1e12, 2),
                             frac_flops=round(flops / t / 1e12 / tf, 3), frac_hbm=round(byts / t / 1e12 / hbm, 3),
                             vs_cublas=round(tc / t, 2)))
            print(json.dumps(rows[-1]), flush=True)
    # attention: decode batch 64 at ~1400 context; prefill 8 x 1024
    decode_attn_rows(args, cfg, dev, timer, hbm, rows, write=False)
    Hq, Hkv, D = cfg.num_attention_heads // args.tp, cfg.num_key_value_heads // args.tp, cfg.head_dim
    B, L = 8, 1024
    nbps = L // 16
    NB = B * nbps + 1
    kc = torch.randn(NB, Hkv, 16, D, device=dev).bfloat16()
    vc = torch.randn_like(kc)
    tables = torch.arange(B * nbps, device=dev).view(B, nbps).int()
    ctxs = torch.full((B,), L, dtype=torch.int32, device=dev)
    cu = torch.arange(0, (B + 1) * L, L, dtype=torch.int32, device=dev)
    q = torch.randn(B * L, Hq, D, device=dev).bfloat16()
    out = torch.empty_like(q)
    t = timer(lambda: ops.prefill_attention(q, kc, vc, tables, ctxs, cu, L, scale=1 / math.sqrt(D), out=out), args.reps)
    flops = 4.0 * B * L * L / 2 * Hq * D
    rows.append(dict(op="prefill_attn", B=B, L=L, us=round(t * 1e6, 1), tflops=round(flops / t / 1e12, 1),
                     frac_flops=round(flops / t / 1e12 / tf, 3)))
    print(json.dumps(rows[-1]), flush=True)
    if args.json:
        json.dump({"peaks": {"hbm_tbs": hbm, "bf16_tflops": tf, "source": src}, "rows": rows},
                  open(args.json, "w"), indent=1)


if __name__ == "__main__":
    main()
