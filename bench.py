"""Headline benchmark: Qwen3-8B-shaped continuous-batching serving (and FSDP training).

    python bench.py --gpus N --steps K --warmup W           # serving, TP=N
    python bench.py --workload train --gpus N ...           # Qwen3-1.7B FSDP fine-tune step
    python bench.py --workload moe --gpus N ...             # gpt-oss-120b serving, EP=N
    python bench.py --workload flux ...                     # FLUX.1-dev DiT, batch 4, 28 steps
    python bench.py --impl reference ...                    # the reference arm

Serving workload: 64 concurrent requests, prompt lengths
uniform in [512, 2048] with uniform-random token ids, 256 output tokens each
(EOS ignored), paged KV with block 16, random-init N(0, 0.02) bf16 weights of
the Qwen3-8B shape. One "step" is one complete pass of the 64-request workload
through the engine (fresh prompts every pass, prefix caching off, so no work
is reused between passes). ``value`` = output tokens / device-timed seconds
over the K timed passes (CUDA events on the launching stream, barrier +
synchronize on both sides, max over ranks). ``e2e`` re-runs one pass through
the public ``LLM.generate`` call, wall-clocked, with its per-step pinned
host->device inputs and device->host token reads counted.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Qwen3-8B-shape TP8 output tok/s/box; p50 TTFT & TPOT; FSDP train tok/s"

# serving workloads: BASELINE config 2 (dense, TP) and config 3 (MoE, EP)
WORKLOADS = {
    "serve": dict(model="qwen3-8b", num_requests=64, min_prompt=512, max_prompt=2048, output_len=256,
                  desc="Qwen3-8B-shape (36L, h4096, 32q/8kv x128, I12288, V151936)", par="tp",
                  l2="inputs larger than L2: every step streams 16 GB of weights + the KV cache"),
    "moe": dict(model="gpt-oss-120b", num_requests=128, min_prompt=1024, max_prompt=1024, output_len=256,
                desc="gpt-oss-120b-shape (36L, h2880, 64q/8kv x64, 128 experts top-4 MXFP4 I2880, SWA128 "
                     "alternating, sinks, V201088)", par="ep",
                l2="inputs larger than L2: every decode step streams ~5 GB of attention/lm_head weights, "
                   "the routed MXFP4 experts and the KV cache"),
}


def reference_arm(args):
    why = ("reference is a Rust/cargo workspace whose engine crates (rlx, rlx-cuda, rlx-runtime ...) are not "
           "in the tree; pip install of the reference tree fails (no setup.py/pyproject) and there is no cargo")
    print(json.dumps({"impl": "reference", "unavailable": why}))
    return 0


def make_prompts(n, lo, hi, vocab, seed):
    import torch
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, hi + 1, (n,), generator=g).tolist()
    return [torch.randint(0, vocab, (l,), generator=g).tolist() for l in lens]


def init_dist(args):
    import torch
    import torch.distributed as dist
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if ws > 1:
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", rank=rank, world_size=ws, timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, ws, local


def serve(args):
    import torch
    import torch.distributed as dist

    from rlx_models_b200 import ops
    from rlx_models_b200.api import LLM, load
    from rlx_models_b200.runtime.engine import EngineConfig, SamplingParams
    from rlx_models_b200.utils.clocks import ClockSampler

    from rlx_models_b200.config import preset

    W = WORKLOADS[args.workload]
    for key in ("num_requests", "min_prompt", "max_prompt", "output_len"):
        if getattr(args, key) is None:
            setattr(args, key, W[key])
    rank, ws, local = init_dist(args)
    dev = torch.device("cuda", local)
    cfg = preset(W["model"])
    comm = None
    if W["par"] == "tp":
        from rlx_models_b200.parallel.tp import make_tp_comm
        comm = make_tp_comm(args.tp_comm, rank, ws, dev, cfg.rms_norm_eps, max_tokens=args.max_batched_tokens,
                            hidden=cfg.hidden_size)
    ecfg = EngineConfig(max_num_seqs=max(64, args.num_requests), max_batched_tokens=args.max_batched_tokens,
                        max_model_len=args.max_prompt + args.output_len + 16, kv_memory_gb=args.kv_gb,
                        prefix_caching=False, cuda_graphs=True, async_scheduling=bool(args.async_sched),
                        metrics_path=args.engine_metrics if rank == 0 else None)
    llm = load(W["model"], device=dev, tp_rank=rank, tp_size=ws, comm=comm, seed=0, engine_config=ecfg,
               config=cfg)
    eng = llm.engine
    sp = SamplingParams(max_new_tokens=args.output_len, ignore_eos=True, temperature=0.0)
    eng.capture_graphs()

    def barrier():
        if ws > 1:
            dist.barrier()

    def one_pass(seed):
        prompts = make_prompts(args.num_requests, args.min_prompt, args.max_prompt, cfg.vocab_size, seed)
        return eng.generate(prompts, sp)

    for w in range(args.warmup):
        one_pass(1000 + w)
    ops.check_errors(dev)

    stream = torch.cuda.current_stream(dev)
    outs_all = []
    barrier()
    torch.cuda.synchronize(dev)
    n0 = ops.launch_count()
    sampler = ClockSampler(local)
    sampler.start()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for k in range(args.steps):
        outs_all.extend(one_pass(2000 + k))
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    sampler.stop()
    launches = ops.launch_count() - n0
    ms = ev0.elapsed_time(ev1)
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ops.check_errors(dev)
    out_tokens = sum(len(o.token_ids) for o in outs_all)
    value = out_tokens / (ms / 1e3)
    ttft = statistics.median(o.ttft for o in outs_all) * 1e3
    tpot = statistics.median(o.tpot for o in outs_all) * 1e3

    # end to end through the public API: one pass, wall clock, bytes counted
    h0, d0 = eng.stats["h2d_bytes"], eng.stats["d2h_bytes"]
    s0 = eng.stats["steps"]
    prompts = make_prompts(args.num_requests, args.min_prompt, args.max_prompt, cfg.vocab_size, 3000)
    barrier()
    torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    e2e_outs = llm.generate(prompts, sp)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_s = time.perf_counter() - t0
    if ws > 1:
        t = torch.tensor([e2e_s], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    nsteps = max(1, eng.stats["steps"] - s0)
    e2e_val = sum(len(o.token_ids) for o in e2e_outs) / e2e_s
    clocks = sampler.summary()
    if args.profile_steps > 0:
        profile_decode(args, eng, cfg, sp, rank, dev)
    res = {
        "metric": METRIC if args.workload == "serve" else f"gpt-oss-120b-shape EP output tok/s (part of: {METRIC})",
        "value": round(value, 1), "unit": "output tok/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 2), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: uniform-random token ids (seeded, fresh per pass), random-init N(0,0.02) weights",
        "config": {"model": W["desc"],
                   "global_batch": args.num_requests, "seq_len": f"prompt U[{args.min_prompt},{args.max_prompt}]"
                   f" + {args.output_len} out", "parallelism": f"{W['par']}{ws}",
                   "tp_comm": args.tp_comm if (ws > 1 and W["par"] == "tp") else None, "kv_block": 16,
                   "async_scheduling": bool(args.async_sched),
                   "max_batched_tokens": args.max_batched_tokens, "l2": W["l2"],
                   "step": f"one full {args.num_requests}-request serving pass"},
        "ttft_p50_ms": round(ttft, 1), "tpot_p50_ms": round(tpot, 2),
        "clocks": clocks,
        "e2e": {"value": round(e2e_val, 1), "unit": "output tok/s via LLM.generate (wall clock)",
                "h2d_bytes_per_step": int((eng.stats["h2d_bytes"] - h0) / nsteps),
                "d2h_bytes_per_step": int((eng.stats["d2h_bytes"] - d0) / nsteps),
                "engine_steps": nsteps},
        "gpu_launches": int(launches),
        "impl": "ours",
    }
    if rank == 0:
        print(json.dumps(res))
    if ws > 1:
        eng.graphs.clear()
        torch.cuda.synchronize(dev)
        dist.destroy_process_group()
    return 0


def profile_decode(args, eng, cfg, sp, rank, dev):
    """Per-kernel device times of ``--profile-steps`` decode steps (torch profiler /
    CUPTI, CUDA graphs off so every kernel is listed), one JSON file per rank.
    Every rank runs the same steps, so collectives stay matched."""
    import dataclasses

    import torch

    from rlx_models_b200.utils.trace import profile
    prompts = make_prompts(args.num_requests, args.min_prompt, args.max_prompt, cfg.vocab_size, 4000)
    for p in prompts:
        eng.add_request(p, sp)
    while eng.stats["graph_steps"] == 0 or eng.sched.num_waiting() > 0:
        eng.step()
        if eng.sched.num_waiting() == 0 and all(len(st.tokens) > 0 for st in eng.requests.values()):
            break
    saved = eng.cfg
    eng.cfg = dataclasses.replace(saved, cuda_graphs=False)
    rows = profile(eng.step, steps=args.profile_steps, warmup=2, top=40)
    eng.cfg = saved
    while eng.has_unfinished():
        eng.step()
    torch.cuda.synchronize(dev)
    out = args.profile_out or "profile_decode"
    with open(f"{out}.rank{rank}.json", "w") as f:
        json.dump({"steps": args.profile_steps, "rows": rows}, f, indent=1)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="serve", choices=["serve", "moe", "train", "flux"])
    ap.add_argument("--num-requests", type=int, default=None)
    ap.add_argument("--min-prompt", type=int, default=None)
    ap.add_argument("--max-prompt", type=int, default=None)
    ap.add_argument("--output-len", type=int, default=None)
    ap.add_argument("--max-batched-tokens", type=int, default=8192)
    ap.add_argument("--kv-gb", type=float, default=40.0)
    ap.add_argument("--micro-batch", type=int, default=4, help="train: sequences per micro-step per rank")
    ap.add_argument("--act-ckpt", type=int, default=0,
                    help="train: 1 = recompute each layer in backward (0 fits: activations of 4 x 4096 tokens ~70 GB)")
    ap.add_argument("--grad-reduce", default="push", choices=["push", "nccl"],
                    help="train: FSDP gradient reduce-scatter by NVLink push or NCCL")
    ap.add_argument("--async-sched", type=int, default=1,
                    help="serving: 1 = schedule / launch step n+1 while step n runs (default), 0 = synchronous loop")
    ap.add_argument("--engine-metrics", default=None, help="serving: write per-step engine metrics (JSONL) here")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="serving: after the timed passes, profile this many eager decode steps per rank")
    ap.add_argument("--profile-out", default=None, help="serving: path prefix of the per-rank profile JSON")
    ap.add_argument("--tp-comm", default="pull", choices=["nccl", "fused", "pull"],
                    help="pull (default): decode steps read every rank's GEMM partial over NVLink in one kernel "
                         "with the residual add + RMSNorm, prefill on NCCL; nccl: NCCL all-reduce baseline; "
                         "fused: GEMM->reduce-scatter push + norm + all-gather over NVLink")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return reference_arm(args)
    if args.workload == "flux":
        from rlx_models_b200.bench.bench_flux import bench_flux
        return bench_flux(args)
    if args.workload == "train":
        from rlx_models_b200.train.bench_train import bench_train
        return bench_train(args)
    return serve(args)


if __name__ == "__main__":
    sys.exit(main())
