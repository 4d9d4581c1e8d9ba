"""Time one decode step (CUDA-graph replay) of a model at a given batch/context.

    python -m rlx_models_b200.bench.decode_step [--model qwen3-8b] [--batch 64] [--ctx 1400] [--iters 20]

Prefills ``batch`` random prompts of ``ctx`` tokens through the engine, then
times ``iters`` replays of the captured decode graph with CUDA events (device
time per step), and reports the weight + KV bytes per step and the achieved
fraction of measured HBM bandwidth. With ``--replays N`` it only replays N
times (for an ncu launch list of one step).

``--tp-emulate N`` builds rank 0 of an N-way tensor-parallel model on this one
GPU with no communicator (every row-parallel reduction is local): the step
then times exactly the compute a TP=N rank does per decode step (its weight
and KV shards, its kernels and launches), so a multi-GPU step time minus this
one is the cost of the collectives. ``--breakdown K`` adds a per-kernel table
of K eager steps (torch profiler; run with B200_PDL=0 so kernel durations do
not include waiting for their predecessor).
"""
from __future__ import annotations

import argparse
import json
import os

import torch


def resident_weight_bytes(model) -> int:
    """Bytes of every distinct CUDA tensor reachable from ``model``'s
    attributes (the weights as stored: bf16, packed MXFP4 blocks + scales),
    except an untied input embedding, of which a decode step reads only the
    batch's rows."""
    seen, total = set(), 0
    skip = set()
    emb, head = getattr(model, "embed", None), getattr(model, "lm_head", None)
    if torch.is_tensor(emb) and not (torch.is_tensor(head) and head.data_ptr() == emb.data_ptr()):
        skip.add(emb.data_ptr())
    stack, visited = [model], set()
    while stack:
        o = stack.pop()
        if id(o) in visited:
            continue
        visited.add(id(o))
        if torch.is_tensor(o):
            if o.is_cuda and o.data_ptr() not in seen and o.data_ptr() not in skip:
                seen.add(o.data_ptr())
                total += o.untyped_storage().nbytes()
        elif isinstance(o, (list, tuple)):
            stack.extend(o)
        elif isinstance(o, dict):
            stack.extend(o.values())
        elif not isinstance(o, type) and type(o).__module__.startswith("rlx_models_b200"):
            if hasattr(o, "__dict__"):
                stack.extend(vars(o).values())
            for c in type(o).__mro__:
                stack.extend(getattr(o, n, None) for n in getattr(c, "__slots__", ()))
    return total


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=1400)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--replays", type=int, default=0)
    ap.add_argument("--tp-emulate", type=int, default=1)
    ap.add_argument("--breakdown", type=int, default=0)
    args = ap.parse_args()
    from .. import ops
    from ..api import load
    from ..config import preset
    from ..runtime.engine import EngineConfig, SamplingParams
    from .bench_ops import peaks

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = preset(args.model)
    ecfg = EngineConfig(max_num_seqs=max(64, args.batch), max_batched_tokens=8192, max_model_len=args.ctx + 64,
                        kv_memory_gb=40, prefix_caching=False)
    tp = args.tp_emulate
    llm = load(args.model, device=dev, engine_config=ecfg, config=cfg, tp_rank=0, tp_size=tp, comm=None)
    eng = llm.engine
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (args.ctx,), generator=g).tolist() for _ in range(args.batch)]
    sp = SamplingParams(max_new_tokens=48, ignore_eos=True)
    for p in prompts:
        eng.add_request(p, sp)
    # run until every sequence is decoding
    while True:
        eng.step()
        if eng.stats["graph_steps"] > 0:
            break
    key = next(k for k in eng.graphs if k[1])
    g_, out, n_launch = eng.graphs[key]
    torch.cuda.synchronize(dev)
    if args.replays:
        torch.cuda.nvtx.range_push("decode_replay")
        for _ in range(args.replays):
            g_.replay()
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_pop()
        print("replayed", args.replays, "launches/step", n_launch)
        return
    for _ in range(3):
        g_.replay()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    for _ in range(args.iters):
        g_.replay()
    ev[1].record()
    torch.cuda.synchronize(dev)
    ms = ev[0].elapsed_time(ev[1]) / args.iters
    ops.check_errors(dev)
    breakdown = None
    if args.breakdown:
        import dataclasses
        from ..utils.trace import profile
        eng.cfg = dataclasses.replace(eng.cfg, cuda_graphs=False)
        breakdown = profile(eng.step, steps=args.breakdown, warmup=1, top=16)
    # weights as stored on this rank (bf16, packed MXFP4 experts); for an MoE every
    # expert counts, an upper bound once a step routes to fewer than all of them
    wbytes = resident_weight_bytes(llm.engine.model)
    kv_bytes = 2 * 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * cfg.head_dim * args.batch * (args.ctx + 1) / tp
    hbm, _, src = peaks()
    ach = (wbytes + kv_bytes) / (ms * 1e-3) / 1e12
    if breakdown is not None:
        for r in breakdown:
            r["us_per_step"] = round(r["device_us_total"] / args.breakdown, 1)
            r["calls_per_step"] = r["calls"] // args.breakdown
            r["name"] = r["name"][:80]
            for k in ("device_us_total", "calls"):
                r.pop(k)
    print(json.dumps({"model": args.model, "tp_emulate": tp, "breakdown": breakdown,
                      "batch": key[0], "ctx": args.ctx, "ms_per_step": round(ms, 3),
                      "launches_per_step": n_launch, "weight_gb": round(wbytes / 1e9, 2),
                      "kv_gb": round(kv_bytes / 1e9, 2), "achieved_tbs": round(ach, 2),
                      "frac_hbm": round(ach / hbm, 3), "peak_source": src}))


if __name__ == "__main__":
    main()
