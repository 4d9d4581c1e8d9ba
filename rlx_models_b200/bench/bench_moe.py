"""gpt-oss MoE block microbenchmark (one layer, one GPU) with roofline fractions.

    python -m rlx_models_b200.bench.bench_moe [--ep 1] [--tokens 128 8192] [--json out.json]
    python -m rlx_models_b200.bench.bench_moe --only gate_up --tokens 128 --iters 3   # plain launches for ncu

Times, per token count, each kernel of the routed expert block (router GEMM,
top-k, align, gather, grouped MXFP4 gate/up GEMM with clamped SwiGLU, grouped
down GEMM, combine) and the whole block, graph-replayed with L2 flushed before
every repetition. Weights are random MXFP4 codes with E8M0 scales 2^-9..2^-7
in the tiled layout the model uses; router logits N(0, 1)-like (near-uniform
expert load). Roofline per grouped GEMM: max(weight bytes of the experts that
received tokens / HBM, FLOPs / bf16 tensor peak), both measured peaks.
"""
from __future__ import annotations

import argparse
import json

import torch

from ..config import gpt_oss_120b
from ..ops._ext import ext, scratch
from .. import ops
from ..quant.mxfp4 import tile_mxfp4
from .bench_ops import Timer, peaks
from ..models.moe import token_tile


def build_layer(cfg, E_l, dev, seed=0):
    H, I = cfg.hidden_size, cfg.moe_intermediate_size
    g = torch.Generator(device=dev).manual_seed(seed)

    def codes(n, k):
        return torch.empty(E_l, n, k // 2, dtype=torch.uint8, device=dev).random_(0, 256, generator=g)

    def scales(n, k):
        return torch.empty(E_l, n, k // 32, dtype=torch.uint8, device=dev).random_(118, 121, generator=g)

    L = dict(router_w=(torch.randn(cfg.num_experts, H, device=dev, generator=g) * 0.02).bfloat16(),
             router_b=torch.zeros(cfg.num_experts, device=dev, dtype=torch.bfloat16),
             gu=tile_mxfp4(codes(2 * I, H), scales(2 * I, H)),
             gu_b=(torch.randn(E_l, 2 * I, device=dev, generator=g) * 0.02).bfloat16(),
             dn=tile_mxfp4(codes(H, I), scales(H, I)),
             dn_b=(torch.randn(E_l, H, device=dev, generator=g) * 0.02).bfloat16())
    return L


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ep", type=int, default=1, help="experts held = 128 / ep (this GPU's share)")
    ap.add_argument("--tokens", type=int, nargs="+", default=[128, 8192])
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--json", default=None)
    ap.add_argument("--only", default=None, choices=[None, "gate_up", "down"])
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = gpt_oss_120b()
    H, I, E, k = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts, cfg.num_experts_per_tok
    E_l = E // args.ep
    L = build_layer(cfg, E_l, dev)
    hbm, tf, src = peaks()
    timer = Timer(dev)
    st = scratch(dev).status
    results = []
    for T in args.tokens:
        n = T * k
        bt = token_tile(n, E)
        x = torch.randn(T, H, device=dev).bfloat16()
        logits = torch.empty(T, E, device=dev, dtype=torch.float32)
        experts = torch.empty(T, k, dtype=torch.int32, device=dev)
        weights = torch.empty(T, k, dtype=torch.float32, device=dev)
        meta = torch.empty(2 * E_l + 2, dtype=torch.int32, device=dev)
        tiles = torch.empty(4 * (n // bt + E_l + 1), dtype=torch.int32, device=dev)
        perm = torch.empty(n, dtype=torch.int32, device=dev)
        inv = torch.empty(n, dtype=torch.int32, device=dev)
        cur = torch.empty(E_l, dtype=torch.int32, device=dev)
        a = torch.empty(n, H, dtype=torch.float16, device=dev)
        gu = torch.empty(n, I, dtype=torch.float16, device=dev)
        dn = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        e_lo = 0
        steps = {
            "router": lambda: ops.linear(x, L["router_w"], bias=L["router_b"], out=logits, out_dtype=torch.float32),
            "route_topk": lambda: ext().moe_route(logits, k, False, True, experts, weights),
            "align": lambda: ext().moe_align(experts, E_l, e_lo, E_l, bt, meta, tiles, perm, inv, cur),
            "gather": lambda: ext().moe_gather(x, perm, meta, E_l, k, a),
            "gate_up": lambda: ext().moe_gemm(a, *L["gu"], 2 * I, L["gu_b"], None, perm, meta, tiles, gu, True,
                                              7.0, 1.702, bt, st),
            "down": lambda: ext().moe_gemm(gu, *L["dn"], H, L["dn_b"], weights.view(-1), perm, meta, tiles, dn,
                                           False, 0.0, 0.0, bt, st),
            "combine": lambda: ext().moe_combine(dn, inv, k, out, False),
        }
        for f in steps.values():  # routing state for the per-kernel timings
            f()
        torch.cuda.synchronize()
        ops.check_errors(dev)
        if args.only:
            for _ in range(args.iters):
                steps[args.only]()
            torch.cuda.synchronize()
            ops.check_errors(dev)
            print(json.dumps({"only": args.only, "tokens": T, "bt": bt, "ok": True}))
            continue
        counts = meta[1:E_l + 1].cpu()
        hit = int((counts > 0).sum())
        local_rows = int(counts.sum())
        row = {"tokens": T, "bt": bt, "experts_hit": hit, "local_rows": local_rows, "us": {}}
        for name, f in steps.items():
            row["us"][name] = round(timer(f, reps=args.reps) * 1e6, 2)
        row["us"]["block"] = round(timer(lambda: [f() for f in steps.values()], reps=args.reps) * 1e6, 2)
        wb_gu = hit * L["gu"][0][0].numel()
        wb_dn = hit * L["dn"][0][0].numel()
        for name, wb, N, K in (("gate_up", wb_gu, 2 * I, H), ("down", wb_dn, H, I)):
            t = row["us"][name] * 1e-6
            flops = 2.0 * local_rows * N * K
            roof = max(wb / (hbm * 1e12), flops / (tf * 1e12))
            row[name] = {"weight_GB": round(wb / 1e9, 3), "TBps": round(wb / t / 1e12, 2) if t else None,
                         "TFLOPs": round(flops / t / 1e12, 1) if t else None,
                         "frac_of_roofline": round(roof / t, 3) if t else None}
        results.append(row)
        print(json.dumps(row), flush=True)
    if args.json and not args.only:
        json.dump({"peaks": {"hbm_TBps": hbm, "bf16_TFLOPs": tf, "source": src}, "ep": args.ep,
                   "rows": results}, open(args.json, "w"), indent=1)


if __name__ == "__main__":
    main()
