"""Same-box library baseline for the serving benchmark: vLLM.

    python -m rlx_models_b200.bench.vllm_baseline [--tp N] [--steps K] [--warmup W]

Runs the headline serving workload (Qwen3-8B shape, 64 concurrent requests,
prompts U[512, 2048] of seeded random token ids, 256 output tokens each with
EOS ignored, paged KV with 16-token blocks, prefix caching off, 8192-token
step budget, bf16, random weights) through vLLM's offline ``LLM.generate``
with ``load_format="dummy"`` (no checkpoint), tensor-parallel over N GPUs of
this box. vLLM runs cuBLAS / cuDNN / FlashInfer / FlashAttention kernels and
NCCL collectives: it is the library-and-NCCL arm the serving numbers of this
package are compared with on identical hardware. Timing is the wall clock of
``generate`` after ``torch.cuda.synchronize`` on both sides (vLLM runs its
own workers; their device timelines are not exposed), averaged over K passes
after W warm-up passes with fresh prompts each pass.

Prints one JSON line with ``"impl": "vllm"``, or ``"unavailable"`` with the
reason when vLLM cannot start.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import tempfile
import time


def qwen3_8b_config_dir() -> str:
    d = tempfile.mkdtemp(prefix="qwen3_8b_shape_")
    cfg = {
        "architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "vocab_size": 151936, "hidden_size": 4096,
        "intermediate_size": 12288, "num_hidden_layers": 36, "num_attention_heads": 32, "num_key_value_heads": 8,
        "head_dim": 128, "rms_norm_eps": 1e-6, "rope_theta": 1000000.0, "max_position_embeddings": 40960,
        "tie_word_embeddings": False, "hidden_act": "silu", "attention_bias": False, "torch_dtype": "bfloat16",
        "bos_token_id": 151643, "eos_token_id": 151645,
    }
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    return d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--num-requests", type=int, default=64)
    ap.add_argument("--min-prompt", type=int, default=512)
    ap.add_argument("--max-prompt", type=int, default=2048)
    ap.add_argument("--output-len", type=int, default=256)
    args = ap.parse_args()
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")
    try:
        import torch
        from vllm import LLM, SamplingParams
        from vllm.inputs import TokensPrompt
        llm = LLM(model=qwen3_8b_config_dir(), skip_tokenizer_init=True, load_format="dummy", dtype="bfloat16",
                  tensor_parallel_size=args.tp, enable_prefix_caching=False, max_num_seqs=args.num_requests,
                  max_num_batched_tokens=8192, block_size=16, gpu_memory_utilization=0.85, seed=0,
                  max_model_len=args.max_prompt + args.output_len + 16)
    except Exception as e:  # pragma: no cover - depends on the box
        print(json.dumps({"impl": "vllm", "unavailable": f"{type(e).__name__}: {e}"[:300]}))
        return 0
    sp = SamplingParams(max_tokens=args.output_len, ignore_eos=True, temperature=0.0, detokenize=False)

    def prompts(seed):
        g = torch.Generator().manual_seed(seed)
        lens = torch.randint(args.min_prompt, args.max_prompt + 1, (args.num_requests,), generator=g).tolist()
        return [TokensPrompt(prompt_token_ids=torch.randint(0, 151936, (n,), generator=g).tolist()) for n in lens]

    for w in range(args.warmup):
        llm.generate(prompts(1000 + w), sp, use_tqdm=False)
    times, toks, ttft, tpot = [], 0, [], []
    for k in range(args.steps):
        ps = prompts(2000 + k)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        outs = llm.generate(ps, sp, use_tqdm=False)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
        for o in outs:
            n = len(o.outputs[0].token_ids)
            toks += n
            m = getattr(o, "metrics", None)
            if m is not None and getattr(m, "first_token_time", None) and getattr(m, "arrival_time", None):
                ttft.append((m.first_token_time - m.arrival_time) * 1e3)
                if getattr(m, "last_token_time", None) and n > 1:
                    tpot.append((m.last_token_time - m.first_token_time) * 1e3 / (n - 1))
    total = sum(times)
    res = {"impl": "vllm", "metric": "Qwen3-8B-shape output tok/s (vLLM, same workload)",
           "value": round(toks / total, 1), "unit": "output tok/s", "n_gpus": args.tp, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(total / args.steps * 1e3, 1), "dtype": "bf16",
           "timing": "wall clock of LLM.generate between cuda synchronizes",
           "config": {"model": "Qwen3-8B-shape, dummy weights", "global_batch": args.num_requests,
                      "seq_len": f"prompt U[{args.min_prompt},{args.max_prompt}] + {args.output_len} out",
                      "parallelism": f"tp{args.tp}", "vllm": __import__("vllm").__version__}}
    if ttft:
        res["ttft_p50_ms"] = round(statistics.median(ttft), 1)
    if tpot:
        res["tpot_p50_ms"] = round(statistics.median(tpot), 2)
    print(json.dumps(res))
    return 0


if __name__ == "__main__":
    sys.exit(main())
