"""Matmul benchmark at model shapes: bf16 dense (this package's tcgen05 GEMM
vs cuBLAS through torch.matmul), the same with the bias + ReLU epilogue, and
the MXFP4 weight-only dense linear (4-bit weights streamed, E2M1 expanded in
TMEM), with achieved TFLOP/s / TB/s against the measured peaks.

    python -m rlx_models_b200.bench.bench_matmul [--model qwen3-8b] [--M 1 64 2048 8192] [--json out.json]

The reference's bench_matmul_rlx measures dense and dequantising matmuls
(+ bias + ReLU) against cuBLAS; this is its counterpart.
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import ops
from ..config import preset
from ..quant.mxfp4 import quantize_mxfp4, tile_mxfp4
from .bench_ops import Timer, peaks


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--M", type=int, nargs="+", default=[1, 64, 2048, 8192])
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = preset(args.model)
    H, I = cfg.hidden_size, cfg.intermediate_size
    shapes = [("qkv", cfg.q_size + 2 * cfg.kv_size, H), ("o_proj", H, cfg.q_size), ("gate_up", 2 * I, H),
              ("down", H, I)]
    hbm, tf, src = peaks()
    timer = Timer(dev)
    rows = []
    for name, N, K in shapes:
        w = (torch.randn(N, K, device=dev) * 0.02).bfloat16()
        b = (torch.randn(N, device=dev) * 0.02).bfloat16()
        blocks, scales = quantize_mxfp4(w.float().view(1, N, K))
        wt, rexp = tile_mxfp4(blocks, scales)
        for M in args.M:
            x = torch.randn(M, K, device=dev).bfloat16()
            out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            t_ours = timer(lambda: ops.linear(x, w, out=out), args.reps)
            t_cub = timer(lambda: torch.matmul(x, w.t()), args.reps)
            t_relu = timer(lambda: ops.linear(x, w, bias=b, relu=True, out=out), args.reps)
            t_cub_relu = timer(lambda: torch.relu(torch.addmm(b, x, w.t())), args.reps)
            t_q = timer(lambda: ops.linear_mxfp4(x, wt, rexp, N, out=out), args.reps)
            fl = 2.0 * M * N * K
            r = dict(op=name, M=M, N=N, K=K, us_ours=round(t_ours * 1e6, 1), us_cublas=round(t_cub * 1e6, 1),
                     us_bias_relu=round(t_relu * 1e6, 1), us_cublas_bias_relu=round(t_cub_relu * 1e6, 1),
                     us_mxfp4=round(t_q * 1e6, 1), tflops_ours=round(fl / t_ours / 1e12, 1),
                     vs_cublas=round(t_cub / t_ours, 2), mxfp4_weight_TBps=round(wt.numel() / t_q / 1e12, 2),
                     bf16_weight_TBps=round(2 * N * K / t_ours / 1e12, 2))
            rows.append(r)
            print(json.dumps(r), flush=True)
    ops.check_errors(dev)
    if args.json:
        json.dump({"peaks": {"hbm_TBps": hbm, "bf16_TFLOPs": tf, "source": src}, "rows": rows},
                  open(args.json, "w"), indent=1)


if __name__ == "__main__":
    main()
