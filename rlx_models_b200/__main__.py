"""Command line: ``python -m rlx_models_b200 <command>``.

    inspect PATH                  config + tensor table of a checkpoint directory (no GPU)
    run --model M --prompt TEXT   load and generate (greedy unless --temperature)
    serve --model M [--port P]    OpenAI-compatible HTTP server
    bench [bench.py args]         the repository benchmark
    train --model M --data F      fine-tune on a JSONL dataset (train.data)

``M`` is a checkpoint directory, an HF id in the offline cache (``org/name``,
optionally ``org/name:QUANT@rev``) or a named shape (``qwen3-0.6b``, ...).

Reference: rlx-cli (`rlx-inspect`), the per-family ``bin/`` runners and
rlx-serve's server binary.
"""
from __future__ import annotations

import argparse
import json
import os
import sys


def cmd_inspect(a):
    from .config import DecoderConfig
    from .weights.safetensors_io import Checkpoint
    path = a.path
    out = {}
    cfgp = os.path.join(path, "config.json")
    if os.path.exists(cfgp):
        with open(cfgp) as f:
            raw = json.load(f)
        out["model_type"] = raw.get("model_type")
        try:
            c = DecoderConfig.from_hf_dict(raw)
            out["config"] = {k: getattr(c, k) for k in ("hidden_size", "num_hidden_layers", "num_attention_heads",
                                                        "num_key_value_heads", "head_dim", "intermediate_size",
                                                        "vocab_size", "num_experts")}
        except Exception as e:  # non-decoder configs
            out["config_error"] = str(e)
    ck = Checkpoint(path)
    names = sorted(ck.keys())
    total = 0
    rows = []
    for n in names:
        dtype, shape = ck.info(n)
        cnt = 1
        for s in shape:
            cnt *= s
        total += cnt
        rows.append((n, dtype, list(shape)))
    out["tensors"] = len(names)
    out["parameters"] = total
    print(json.dumps(out, indent=1, default=str))
    if a.tensors:
        for n, d, s in rows[:a.limit]:
            print(f"{n:70s} {str(d):10s} {s}")
    return 0


def _run_config(a):
    """The --config file's RunConfig (or an empty one); applies its knob
    overrides and prints the knob table with --show-knobs."""
    from . import settings
    rc = settings.load_run_config(a.config) if getattr(a, "config", None) else settings.RunConfig()
    rc.apply_kernel_overrides()
    if getattr(a, "show_knobs", False):
        print(settings.describe(), file=sys.stderr)
    return rc


def _explicit(a, ap_defaults: dict, mapping: dict) -> dict:
    """EngineConfig / TrainConfig fields given explicitly on the command line
    (values that differ from the parser defaults), as keyword arguments."""
    return {field: getattr(a, dest) for dest, field in mapping.items() if getattr(a, dest) != ap_defaults.get(dest)}


def cmd_run(a):
    from .api import load
    from .runtime.engine import SamplingParams
    rc = _run_config(a)
    base = {"max_num_seqs": 8, "max_model_len": a.max_model_len, "kv_memory_gb": a.kv_gb}
    cli = _explicit(a, a._defaults, {"max_model_len": "max_model_len", "kv_gb": "kv_memory_gb",
                                     "kv_cache_dtype": "kv_cache_dtype"})
    llm = load(a.model or rc.model, engine_config=rc.engine_config(**{**{k: v for k, v in base.items()
                                                                         if k not in rc.serve}, **cli}))
    tok = llm.tokenizer
    if a.ids:
        ids = [int(x) for x in a.ids.split(",")]
    else:
        from .tokenizer import ByteTokenizer
        tok = tok or ByteTokenizer()
        ids = tok.encode(a.prompt)
    sp = SamplingParams(max_new_tokens=a.max_tokens, temperature=a.temperature, top_p=a.top_p, top_k=a.top_k,
                        seed=a.seed, ignore_eos=a.ignore_eos)
    out = llm.generate([ids], sp)[0]
    res = {"token_ids": out.token_ids, "finish_reason": out.finish_reason, "ttft_ms": round(out.ttft * 1e3, 2),
           "tpot_ms": round(out.tpot * 1e3, 3)}
    if tok is not None:
        res["text"] = tok.decode(out.token_ids)
    print(json.dumps(res))
    return 0


def cmd_serve(a):
    from .api import load
    from .serve.openai_server import serve
    rc = _run_config(a)
    base = {"max_num_seqs": a.max_num_seqs, "max_model_len": a.max_model_len, "kv_memory_gb": a.kv_gb}
    cli = _explicit(a, a._defaults, {"max_num_seqs": "max_num_seqs", "max_model_len": "max_model_len",
                                     "kv_gb": "kv_memory_gb", "kv_cache_dtype": "kv_cache_dtype"})
    model = a.model or rc.model
    llm = load(model, engine_config=rc.engine_config(**{**{k: v for k, v in base.items() if k not in rc.serve},
                                                        **cli}))
    embedder = None
    if a.embed_model:  # an encoder checkpoint behind /v1/embeddings
        from .api import load_embedder
        embedder = load_embedder(a.embed_model)
    transcriber = None
    if a.asr_model:  # a Whisper checkpoint behind /v1/audio/transcriptions
        from .api import load_transcriber
        transcriber = load_transcriber(a.asr_model)
    serve(llm, a.host, a.port, model_name=model, embedder=embedder, transcriber=transcriber)
    return 0


def cmd_profile(a):
    """Profile engine steps: prefill the requests, then ``--steps`` decode
    steps under the torch profiler; prints the top kernels by device time and
    writes a Chrome trace. Decode CUDA graphs are off by default so every
    kernel shows up on its own."""
    import torch

    from .api import load
    from .runtime.engine import EngineConfig, SamplingParams
    from .utils.trace import enable_nvtx, profile
    enable_nvtx(True)
    llm = load(a.model, engine_config=EngineConfig(max_num_seqs=max(8, a.batch), max_model_len=a.prompt_len + 512,
                                                   kv_memory_gb=a.kv_gb, cuda_graphs=a.graphs))
    eng = llm.engine
    g = torch.Generator().manual_seed(0)
    V = llm.config.vocab_size
    for _ in range(a.batch):
        eng.add_request(torch.randint(0, V, (a.prompt_len,), generator=g).tolist(),
                        SamplingParams(max_new_tokens=a.steps + 64, ignore_eos=True))
    while eng.stats["steps"] < 1 or any(len(st.tokens) == 0 for st in eng.requests.values()):
        eng.step()  # prefill
    rows = profile(eng.step, steps=a.steps, warmup=2, trace_path=a.trace)
    for r in rows:
        print(json.dumps(r))
    return 0


def cmd_bench(rest):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.argv = ["bench.py"] + rest
    import bench
    return bench.main()


def cmd_train(a):
    from .train.data import train_from_jsonl
    a.run_config = _run_config(a)
    a.model = a.model or a.run_config.model
    return train_from_jsonl(a)


def cmd_knobs(a):
    """Print every environment knob with its value and where it came from."""
    _run_config(a)
    from . import settings
    print(settings.describe())
    return 0


def cmd_scan(a):
    """List (or resolve) locally cached checkpoints: weights/discover.py."""
    from .weights.discover import resolve, scan
    if a.resolve:
        p = resolve(a.query or "")
        print(p or "")
        return 0 if p else 1
    for h in scan(query=a.query):
        print(f"{h.source:9s} {h.fmt:12s} {h.name}  ->  {h.path}")
    return 0


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "bench":
        return cmd_bench(argv[1:])
    ap = argparse.ArgumentParser(prog="python -m rlx_models_b200")
    sub = ap.add_subparsers(dest="cmd", required=True)
    p = sub.add_parser("scan", help="list weights found in local caches (LM Studio, Ollama, HF, RLX_WEIGHTS_*)")
    p.add_argument("query", nargs="?", default=None)
    p.add_argument("--resolve", action="store_true", help="print only the path a query resolves to")
    p = sub.add_parser("inspect")
    p.add_argument("path")
    p.add_argument("--tensors", action="store_true")
    p.add_argument("--limit", type=int, default=100000)
    for name in ("run", "serve"):
        p = sub.add_parser(name)
        p.add_argument("--model", default=None, help="model id, preset or path (or the config file's 'model')")
        p.add_argument("--config", default=None, help="YAML / JSON run config (settings.RunConfig)")
        p.add_argument("--show-knobs", action="store_true", help="print the knob table at startup")
        p.add_argument("--max-model-len", type=int, default=4096)
        p.add_argument("--kv-gb", type=float, default=8.0)
        p.add_argument("--kv-cache-dtype", default="bf16", choices=["bf16", "fp8"],
                       help="fp8: e4m3 KV pages (half the cache bytes; the decode kernel reads them directly)")
        if name == "run":
            p.add_argument("--prompt", default="Hello")
            p.add_argument("--ids", default=None, help="comma-separated token ids instead of --prompt")
            p.add_argument("--max-tokens", type=int, default=32)
            p.add_argument("--temperature", type=float, default=0.0)
            p.add_argument("--top-p", type=float, default=1.0)
            p.add_argument("--top-k", type=int, default=0)
            p.add_argument("--seed", type=int, default=0)
            p.add_argument("--ignore-eos", action="store_true")
        else:
            p.add_argument("--host", default="127.0.0.1")
            p.add_argument("--port", type=int, default=8000)
            p.add_argument("--max-num-seqs", type=int, default=64)
            p.add_argument("--embed-model", default=None, help="encoder checkpoint served at /v1/embeddings")
            p.add_argument("--asr-model", default=None, help="Whisper checkpoint served at /v1/audio/transcriptions")
    p = sub.add_parser("profile")
    p.add_argument("--model", default="qwen3-0.6b")
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--prompt-len", type=int, default=256)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--kv-gb", type=float, default=4.0)
    p.add_argument("--graphs", action="store_true", help="keep decode CUDA graphs (kernels then appear per graph)")
    p.add_argument("--trace", default="b200_trace.json")
    p = sub.add_parser("knobs", help="print the environment knobs and their values")
    p.add_argument("--config", default=None)
    p = sub.add_parser("train")
    p.add_argument("--model", default=None)
    p.add_argument("--config", default=None, help="YAML / JSON run config (its 'train' section)")
    p.add_argument("--show-knobs", action="store_true")
    p.add_argument("--data", required=True, help="JSONL with 'text', 'prompt'/'completion' or 'input_ids'")
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--seq-len", type=int, default=2048)
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--lr", type=float, default=1e-4)
    p.add_argument("--out", default=None)
    p.add_argument("--lora-rank", type=int, default=0)
    a = ap.parse_args(argv)
    if a.cmd in ("run", "serve", "train"):
        a._defaults = {act.dest: act.default for act in sub.choices[a.cmd]._actions}
    if a.cmd in ("run", "serve", "train") and not (a.model or (a.config and _peek_model(a.config))):
        ap.error(f"{a.cmd}: --model (or a --config file with 'model') is required")
    return {"scan": cmd_scan, "inspect": cmd_inspect, "run": cmd_run, "serve": cmd_serve, "train": cmd_train,
            "profile": cmd_profile, "knobs": cmd_knobs}[a.cmd](a)


def _peek_model(path: str):
    from . import settings
    return settings.load_run_config(path).model


if __name__ == "__main__":
    sys.exit(main())
