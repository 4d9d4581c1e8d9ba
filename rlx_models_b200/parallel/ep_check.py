"""Multi-GPU expert-parallel check and combine microbenchmark (torchrun).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m rlx_models_b200.parallel.ep_check [--bench]

Correctness: a seeded gpt-oss-structured MoE decoder at EP=N with the fused
NVLink combine (parallel/ep.py) must give the EP=1 model's prefill logits bit
for bit and the same greedy generations through the engine (CUDA graphs on);
the NCCL all-reduce combine is checked within bf16 tolerance.

``--bench`` also times one layer's combine at the gpt-oss-120b decode shape
(128 tokens, top-4, hidden 2880) per rank with CUDA events under a CUDA graph,
max over ranks: the fused kernel against the NCCL path it replaces (local
combine, NCCL all-reduce, add + RMSNorm), and reports the fused kernel's
fraction of its NVLink roofline (remote expert-row bytes at the measured
770 GB/s per direction).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist


def check(rank, world, dev):
    from rlx_models_b200 import config as C
    from rlx_models_b200 import ops
    from rlx_models_b200.models.decoder import ForwardBatch
    from rlx_models_b200.models.moe import MoEDecoderLM
    from rlx_models_b200.runtime.engine import EngineConfig, LLMEngine, SamplingParams
    from rlx_models_b200.weights.init import random_weights

    cfg = C.tiny("gpt_oss", hidden_size=512, num_attention_heads=8, num_key_value_heads=2, head_dim=64,
                 num_experts=16, num_experts_per_tok=4, moe_intermediate_size=256, intermediate_size=256,
                 vocab_size=1024, num_hidden_layers=4, sliding_window=16,
                 layer_types=["sliding_attention", "full_attention"] * 2)
    w = random_weights(cfg, seed=11, dtype=torch.bfloat16)
    ref = MoEDecoderLM(cfg, w, device=dev)  # EP=1 on this GPU
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 40, 100, 3)]
    sp = SamplingParams(max_new_tokens=10, ignore_eos=True)
    ecfg = dict(max_num_seqs=8, max_batched_tokens=256, max_model_len=256, num_blocks=128)
    ref_tokens = [o.token_ids for o in LLMEngine(ref, EngineConfig(**ecfg)).generate(prompts, sp)]
    T = 70
    ids = torch.tensor(prompts[2][:T], dtype=torch.int32, device=dev)
    nb = (T + 15) // 16

    def fb():
        return ForwardBatch(input_ids=ids, positions=torch.arange(T, dtype=torch.int32, device=dev),
                            slots=torch.arange(T, dtype=torch.int64, device=dev), num_decode=0,
                            pre_block_tables=torch.arange(nb, dtype=torch.int32, device=dev).view(1, -1),
                            pre_ctx_lens=torch.tensor([T], dtype=torch.int32, device=dev),
                            pre_cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), pre_max_q=T)

    ref_logits = ref.forward(fb(), ref.make_kv_cache(nb))
    ok_all = True
    for kind in ("fused", "nccl"):
        m = MoEDecoderLM(cfg, w, device=dev, ep_rank=rank, ep_size=world, ep_combine=kind)
        lg = m.forward(fb(), m.make_kv_cache(nb))
        exact = bool(torch.equal(lg, ref_logits))
        rel = ((lg.float() - ref_logits.float()).norm() / ref_logits.float().norm()).item()
        eng = LLMEngine(m, EngineConfig(**ecfg))
        toks = [o.token_ids for o in eng.generate(prompts, sp)]
        agree = sum(a == b for a, b in zip(toks, ref_tokens))
        ops.check_errors(dev)
        ok = (exact and agree == len(prompts)) if kind == "fused" else (rel < 2e-2 and
                                                                          all(a[0] == b[0] for a, b in
                                                                              zip(toks, ref_tokens)))
        t = torch.tensor([1.0 if ok else 0.0], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        ok_all &= bool(t.item() == 1.0)
        if rank == 0:
            print(json.dumps({"ep_combine": kind, "world": world, "logits_bitwise_equal": exact,
                              "logits_rel_err": rel, "seqs_equal": agree, "seqs": len(prompts),
                              "graph_steps": eng.stats["graph_steps"], "ok_all_ranks": bool(t.item() == 1.0)}),
                  flush=True)
        eng.graphs.clear()
        torch.cuda.synchronize(dev)
        dist.barrier()
        if m.combiner is not None:
            m.combiner.close()
    return ok_all


def bench(rank, world, dev, T=128, k=4, H=2880, E=128, iters=100):
    from rlx_models_b200 import ops
    from rlx_models_b200.ops._ext import ext
    from rlx_models_b200.parallel.ep import EPCombiner

    e_local = E // world
    g = torch.Generator(device=dev).manual_seed(0)  # same routing on every rank
    experts = torch.randn(T, E, device=dev, generator=g).topk(k, -1).indices.int().contiguous()
    n = T * k
    comb = EPCombiner(rank, world, dev, hidden=H, top_k=k, e_local=e_local, max_tokens=T, num_layers=2, eps=1e-6)
    meta = torch.empty(2 * e_local + 2, dtype=torch.int32, device=dev)
    tiles = torch.empty(4 * (n // 32 + e_local + 1), dtype=torch.int32, device=dev)
    perm = torch.empty(n, dtype=torch.int32, device=dev)
    cur = torch.empty(e_local, dtype=torch.int32, device=dev)
    for p in (0, 1):
        ext().moe_align(experts, e_local, rank * e_local, e_local, 32, meta, tiles, perm, comb.inv[p, :n], cur)
        comb.rows[p].normal_(0, 0.1)
    inv_local = comb.inv[0, :n].clone()
    dn_local = comb.rows[0, :n].clone()
    nw = torch.ones(H, device=dev, dtype=torch.bfloat16)
    h = torch.zeros(T, H, device=dev, dtype=torch.bfloat16)
    torch.cuda.synchronize(dev)
    dist.barrier()

    def fused():
        comb.combine_norm(experts, h, nw)

    def nccl():
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        ext().moe_combine(dn_local, inv_local, k, out, False)
        dist.all_reduce(out)
        ops.rmsnorm(out, nw, 1e-6, residual=h, residual_out=h)

    res = {}
    for name, op in (("fused", fused), ("nccl", nccl)):
        for _ in range(6):
            op()
        torch.cuda.synchronize(dev)
        gr = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            op()
            op()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        dist.barrier()
        with torch.cuda.graph(gr):
            for _ in range(iters):
                op()
        dist.barrier()
        gr.replay()  # warm replay
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        gr.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / iters * 1e3], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name + "_us"] = round(float(t), 2)
        ops.check_errors(dev)
        del gr
        torch.cuda.synchronize(dev)
        dist.barrier()
    remote = float((experts // e_local != rank).sum().item()) * H * 2  # expert rows read over NVLink
    roof_us = remote / 770e9 * 1e6
    res.update(world=world, T=T, k=k, H=H, remote_bytes=int(remote), nvlink_roofline_us=round(roof_us, 2),
               fused_frac_of_roofline=round(roof_us / res["fused_us"], 3))
    comb.close()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--bench", action="store_true")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    ok = check(rank, world, dev)
    if args.bench:
        r = bench(rank, world, dev)
        if rank == 0:
            print(json.dumps({"ep_combine_bench": r}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
