"""The reference's own published Qwen3-0.6B numbers, measured on a B200 with
this framework (same workload shapes, device-timed).

    python -m rlx_models_b200.bench.bench_reference_rows [--json out.json]

Model: Qwen3-0.6B shape (28 layers, hidden 1024, 16 q / 8 kv heads x 128,
SwiGLU 3072, vocab 151936, tied embeddings), random-init weights written as a
Q4_K_M-style GGUF (Q4_K matrices, Q6_K embedding, F32 norms), loaded through
``api.load`` (blocks dequantised on the GPU to bf16; the kernels then run
bf16). Rows (reference value, hardware in parentheses):

  1. single-stream greedy decode at ~140 tokens of context: 51.3 tok/s (M4 Pro)
  2. batched decode, uniform prompts, aggregate tok/s at B = 8 / 16 / 32:
     62 / 91 / 91 (M4 Pro)
  5. prefix-cache TTFT: time to the first token of a 2048-token prompt, cold
     vs with the 2048-token prefix cached: 9.2 s -> 1.2 s (M4 Pro)
  7. long-context retrieval at 16k tokens of context: retrieval ~25 ms, decode
     ~59 tok/s (M4 Pro, HNSW KV store); here single-stream decode at 16k with
     KV-block retrieval (64 top-k + 16 recent + 1 sink blocks) and with full
     attention, plus the device time of one retrieval selection over all
     layers

Each decode row times ``--tokens`` generated tokens per sequence with CUDA
events around ``LLMEngine.generate`` (decode steps run as CUDA graphs),
excluding the prompt's prefill step; TTFT rows are one-request wall clock
through the engine (with a device synchronise).
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile
import time

import torch

REF = {"single_stream_tok_s": 51.3, "batched_tok_s": {8: 62.0, 16: 91.0, 32: 91.0},
       "ttft_2048_cold_s": 9.2, "ttft_2048_cached_s": 1.2, "retrieval_16k_ms": 25.0, "decode_16k_tok_s": 59.0}


def build_gguf(path: str, seed: int = 0):
    from ..config import qwen3_0_6b
    from ..weights.gguf import GGUFWriter, hf_to_gguf_name
    from ..weights.init import random_weights
    cfg = qwen3_0_6b()
    w = random_weights(cfg, seed, device="cuda" if torch.cuda.is_available() else "cpu")
    gw = GGUFWriter(path)
    gw.add("general.architecture", "qwen3")
    for k, v in (("block_count", cfg.num_hidden_layers), ("embedding_length", cfg.hidden_size),
                 ("feed_forward_length", cfg.intermediate_size), ("attention.head_count", cfg.num_attention_heads),
                 ("attention.head_count_kv", cfg.num_key_value_heads), ("attention.key_length", cfg.head_dim),
                 ("context_length", 40960)):
        gw.add(f"qwen3.{k}", int(v))
    gw.add("qwen3.attention.layer_norm_rms_epsilon", float(cfg.rms_norm_eps))
    gw.add("qwen3.rope.freq_base", float(cfg.rope_theta))
    for name, t in w.items():
        kind = "F32" if t.dim() == 1 else ("Q6_K" if "embed_tokens" in name else "Q4_K")
        gw.add_tensor(hf_to_gguf_name(name), t.float(), kind)
    gw.write()
    return cfg


def long_context_rows(gguf: str, tokens: int, ctx: int = 16384) -> list[dict]:
    """Row 7: single-stream decode at ``ctx`` tokens of context with and
    without KV-block retrieval, and one retrieval selection's device time."""
    from ..api import load
    from ..runtime.engine import EngineConfig, SamplingParams
    out = []
    g = torch.Generator().manual_seed(7)
    for kvr in ({"topk_blocks": 64, "window_blocks": 16, "sink_blocks": 1}, None):
        kv_gb = max(8.0, 2.5 * ctx * 28 * 8 * 128 * 4 / 2 ** 30)
        llm = load(gguf, device="cuda", engine_config=EngineConfig(max_num_seqs=2, max_model_len=ctx + tokens + 32,
                                                                    kv_memory_gb=kv_gb, prefix_caching=False,
                                                                    kv_retrieval=kvr, chunk_size=4096))
        eng = llm.engine
        V = llm.config.vocab_size
        eng.capture_graphs(sizes=[1])
        prompt = torch.randint(0, V, (ctx,), generator=g).tolist()
        eng.generate([prompt[:64]], SamplingParams(max_new_tokens=4, ignore_eos=True))  # warm-up
        torch.cuda.synchronize()
        o = eng.generate([prompt], SamplingParams(max_new_tokens=tokens, ignore_eos=True))[0]
        torch.cuda.synchronize()
        name = "with KV-block retrieval" if kvr else "full attention"
        out.append({"row": f"decode tok/s at {ctx} tokens of context, {name}", "value": round(1.0 / o.tpot, 1),
                    "reference": REF["decode_16k_tok_s"], "ratio": round(1.0 / o.tpot / REF["decode_16k_tok_s"], 1)})
        if kvr:
            m = llm.model
            r = m.retrieval
            W = eng.max_blocks_per_seq
            tables = torch.arange(W, dtype=torch.int32, device="cuda")[None]
            ctx_t = torch.tensor([ctx], dtype=torch.int32, device="cuda")
            q = torch.randn(1, m.hq, m.D, device="cuda").bfloat16()
            for _ in range(3):
                for layer in range(len(m.layers)):
                    r.select(layer, q, tables, ctx_t)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for layer in range(len(m.layers)):
                r.select(layer, q, tables, ctx_t)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            out.append({"row": f"retrieval selection at {ctx} tokens, all {len(m.layers)} layers (ms)",
                        "value": round(ms, 3), "reference": REF["retrieval_16k_ms"],
                        "ratio": round(REF["retrieval_16k_ms"] / ms, 1)})
        del llm, eng
        torch.cuda.empty_cache()
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=128)
    ap.add_argument("--long-ctx", type=int, nargs="*", default=[16384],
                    help="contexts for the retrieval rows (row 7 is quoted at 16384)")
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    from ..api import load
    from ..runtime.engine import EngineConfig, SamplingParams
    dev = torch.device("cuda", 0)
    tmp = tempfile.mkdtemp()
    gguf = os.path.join(tmp, "qwen3-0.6b-Q4_K_M.gguf")
    t0 = time.perf_counter()
    build_gguf(gguf)
    t_build = time.perf_counter() - t0
    rows = []
    llm = load(gguf, device=dev, engine_config=EngineConfig(max_num_seqs=64, max_model_len=4608, kv_memory_gb=8,
                                                              prefix_caching=True))
    eng = llm.engine
    V = llm.config.vocab_size
    g = torch.Generator().manual_seed(0)
    eng.capture_graphs()

    def decode_rate(B, prompt_len=12):
        prompts = [torch.randint(0, V, (prompt_len,), generator=g).tolist() for _ in range(B)]
        sp = SamplingParams(max_new_tokens=a.tokens, ignore_eos=True)
        eng.generate(prompts, SamplingParams(max_new_tokens=8, ignore_eos=True))  # warm-up
        # time decode only: the first generated token comes from the prefill step
        torch.cuda.synchronize()
        outs = eng.generate([p + [1] for p in prompts], sp)
        torch.cuda.synchronize()
        tpot = sum(o.tpot for o in outs) / len(outs)  # engine per-token time after the first token
        return B / tpot

    ss = decode_rate(1, prompt_len=128)  # ~140 tokens of context, like the reference's row
    rows.append({"row": "single-stream decode tok/s (Qwen3-0.6B, Q4_K_M GGUF, ctx ~140)", "value": round(ss, 1),
                 "reference": REF["single_stream_tok_s"], "ratio": round(ss / REF["single_stream_tok_s"], 1)})
    for B in (8, 16, 32):
        r = decode_rate(B)
        rows.append({"row": f"batched decode aggregate tok/s, B={B}", "value": round(r, 1),
                     "reference": REF["batched_tok_s"][B], "ratio": round(r / REF["batched_tok_s"][B], 1)})
    prefix = torch.randint(0, V, (2048,), generator=g).tolist()

    def ttft(prompt):
        torch.cuda.synchronize()
        o = eng.generate([prompt], SamplingParams(max_new_tokens=1, ignore_eos=True))[0]
        torch.cuda.synchronize()
        return o.ttft

    cold = ttft(prefix + [5])
    cached = ttft(prefix + [7])  # the 2048-token prefix (128 full blocks) is reused
    rows.append({"row": "TTFT, 2048-token prompt, cold (s)", "value": round(cold, 4), "reference": REF["ttft_2048_cold_s"],
                 "ratio": round(REF["ttft_2048_cold_s"] / cold, 1)})
    rows.append({"row": "TTFT, 2048-token prefix cached (s)", "value": round(cached, 4),
                 "reference": REF["ttft_2048_cached_s"], "ratio": round(REF["ttft_2048_cached_s"] / cached, 1)})
    for n in a.long_ctx:
        rows += long_context_rows(gguf, a.tokens, n)
    meta = {"device": torch.cuda.get_device_name(0), "gguf_build_s": round(t_build, 1),
            "note": "reference values are the reference's published Apple M4 Pro numbers; ratio > 1 = faster here"}
    for r in rows:
        print(json.dumps(r), flush=True)
    print(json.dumps(meta))
    if a.json:
        json.dump({"rows": rows, "meta": meta}, open(a.json, "w"), indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
