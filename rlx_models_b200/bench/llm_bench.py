"""LLM benchmark harness: speed, quality and parity over any model adapter.

    python -m rlx_models_b200.bench.llm_bench speed  --model qwen3-0.6b [--dry-run]
    python -m rlx_models_b200.bench.llm_bench mc     --model <dir> --data mmlu.jsonl [--mode letter|raw]
    python -m rlx_models_b200.bench.llm_bench gsm8k  --model <dir> --data gsm8k.jsonl
    python -m rlx_models_b200.bench.llm_bench ppl    --model <dir> --text file.txt
    python -m rlx_models_b200.bench.llm_bench parity --model <dir> --save-ref ref.pt | --ref ref.pt
    python -m rlx_models_b200.bench.llm_bench all    ... --report LLM_BENCH.md

A model joins through a small adapter with ``logits(ids) -> [T, V]`` and
``generate(ids, n) -> (tokens, ttft_s, total_s)``: ``EngineModel`` (the GPU
engine behind ``api.load``), ``OracleModel`` (the fp32 CPU reference) and
``MockModel`` (weightless, for ``--dry-run``). Speed reports prefill and decode
tok/s, TTFT and peak device memory (host RSS on CPU); quality reuses
``rlx_models_b200.eval`` scoring (letter mode scores one next-token logit per
option letter; raw mode the continuation log-likelihood); parity compares
argmax tokens and logit cosine with a saved reference dump or another model.
Every dimension prints a machine-readable ``LLMBENCH kind=... key=value``
line and a markdown leaderboard row. Without ``--data`` a small built-in
synthetic set is used (and said so): there is no network here.

Reference: crates/rlx-llm-bench (speed.rs `run_speed`, parity.rs, metrics.rs,
mock.rs, README: LLMBENCH lines, JSONL formats, letter / raw MC modes).
"""
from __future__ import annotations

import argparse
import json
import math
import re
import resource
import time
from dataclasses import dataclass, field

import torch

from .. import eval as E


# ---------------------------------------------------------------------------
# model adapters
# ---------------------------------------------------------------------------

class MockModel:
    """Deterministic weightless model: the next token is (last + 1) mod V."""

    name, device = "mock", "cpu"

    def __init__(self, vocab: int = 256):
        self.V = vocab
        self.tokenizer = None

    def logits(self, ids):
        ids = torch.as_tensor(list(ids))
        lg = torch.full((len(ids), self.V), -4.0)
        lg[torch.arange(len(ids)), (ids + 1) % self.V] = 4.0
        return lg

    def generate(self, ids, n):
        t0 = time.perf_counter()
        out = [(ids[-1] + 1 + i) % self.V for i in range(n)]
        t1 = time.perf_counter()
        return out, t1 - t0, t1 - t0


class OracleModel:
    device = "cpu"

    def __init__(self, cfg, weights, name="oracle", tokenizer=None):
        from ..models.oracle import DecoderOracle
        self.m = DecoderOracle(cfg, {k: v.float() for k, v in weights.items()})
        self.name, self.tokenizer = name, tokenizer

    def logits(self, ids):
        return self.m.forward(torch.as_tensor(list(ids)))[0]

    def generate(self, ids, n):
        t0 = time.perf_counter()
        lg, kv = self.m.forward(torch.as_tensor(list(ids)))
        ttft = time.perf_counter() - t0
        out = [int(lg[-1].argmax())]
        for _ in range(n - 1):
            lg, kv = self.m.forward(torch.tensor([out[-1]]), kv)
            out.append(int(lg[-1].argmax()))
        return out, ttft, time.perf_counter() - t0


class EngineModel:
    device = "cuda"

    def __init__(self, llm, name="model"):
        self.llm, self.name, self.tokenizer = llm, name, llm.tokenizer

    def logits(self, ids):
        return self.llm.logits(list(ids))

    def generate(self, ids, n):
        from ..runtime.engine import SamplingParams
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = self.llm.generate([list(ids)], SamplingParams(max_new_tokens=n, ignore_eos=True))[0]
        torch.cuda.synchronize()
        return out.token_ids, out.ttft, time.perf_counter() - t0


# ---------------------------------------------------------------------------
# dimensions
# ---------------------------------------------------------------------------

@dataclass
class Result:
    kind: str
    model: str
    device: str
    fields: dict = field(default_factory=dict)

    def line(self) -> str:
        kv = " ".join(f"{k}={_fmt(v)}" for k, v in self.fields.items())
        return f"LLMBENCH kind={self.kind} model={self.model} device={self.device} {kv}"

    def row(self) -> str:
        return f"| {self.model} | {self.device} | {self.kind} | " + ", ".join(
            f"{k} {_fmt(v)}" for k, v in self.fields.items()) + " |"


def _fmt(v):
    if isinstance(v, float):
        return f"{v:.6g}"
    if isinstance(v, bool):
        return "yes" if v else "no"
    return str(v)


def _peak_mem_mb(device) -> float:
    if device == "cuda" and torch.cuda.is_available():
        return torch.cuda.max_memory_allocated() / 2 ** 20
    return resource.getrusage(resource.RUSAGE_SELF).ru_maxrss / 1024.0


def speed(model, prompt_len: int = 128, gen_len: int = 64, seed: int = 0) -> Result:
    V = getattr(model, "V", None) or 1000
    ids = torch.randint(0, V, (prompt_len,), generator=torch.Generator().manual_seed(seed)).tolist()
    model.logits(ids[:8])  # warm-up
    t0 = time.perf_counter()
    model.logits(ids)
    if model.device == "cuda":
        torch.cuda.synchronize()
    t_pre = time.perf_counter() - t0
    toks, ttft, total = model.generate(ids, gen_len)
    dec = max(1e-9, total - ttft)
    return Result("speed", model.name, model.device, dict(
        prompt_toks=prompt_len, gen_toks=len(toks), prefill_tok_s=prompt_len / max(1e-9, t_pre),
        decode_tok_s=(len(toks) - 1) / dec if len(toks) > 1 else 0.0, ttft_ms=ttft * 1e3,
        peak_mem_mb=_peak_mem_mb(model.device)))


LETTERS = "ABCDEFGHIJ"


def _encode(model, text: str) -> list[int]:
    tok = getattr(model, "tokenizer", None)
    if tok is None:
        return list(text.encode("utf-8"))
    return tok.encode(text)


def load_jsonl(path: str, limit: int | None = None) -> list[dict]:
    rows = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if line:
                rows.append(json.loads(line))
            if limit and len(rows) >= limit:
                break
    return rows


def synthetic_mc(n: int = 8) -> list[dict]:
    """Built-in smoke set (arithmetic facts), used when no --data is given."""
    rows = []
    for i in range(n):
        a, b = 2 + i, 3 + 2 * i
        right = a + b
        choices = [str(right + d) for d in (-1, 0, 1, 2)]
        rows.append({"question": f"What is {a} + {b}?", "choices": choices, "answer": 1})
    return rows


def _answer_index(a) -> int:
    if isinstance(a, int):
        return a
    a = str(a).strip()
    return LETTERS.index(a.upper()) if a and a[0].upper() in LETTERS and len(a) == 1 else int(a)


def multiple_choice(model, rows: list[dict], mode: str = "letter") -> Result:
    """letter: prompt lists lettered options, score the next-token logit of
    each letter at the prompt's end; raw: score log p(choice text | question)."""
    correct = 0
    for r in rows:
        gold = _answer_index(r["answer"])
        if mode == "letter":
            body = r["question"] + "\n" + "\n".join(f"{LETTERS[i]}. {c}" for i, c in enumerate(r["choices"]))
            ids = _encode(model, body + "\nAnswer:")
            lp = torch.log_softmax(model.logits(ids)[-1].float(), -1)
            letter_ids = [_encode(model, " " + LETTERS[i])[-1] for i in range(len(r["choices"]))]
            pred = int(torch.stack([lp[t] for t in letter_ids]).argmax())
        else:
            ctx = _encode(model, r["question"])
            sc = E.multiple_choice(model.logits, ctx, [_encode(model, " " + c) for c in r["choices"]])
            pred = sc.best_norm
        correct += int(pred == gold)
    return Result("mc", model.name, model.device, dict(mode=mode, n=len(rows), accuracy=correct / max(1, len(rows))))


_NUM = re.compile(r"-?\d[\d,]*\.?\d*")


def gsm8k(model, rows: list[dict], max_new_tokens: int = 128, decode=None) -> Result:
    """Generative: greedy answer, the last number in the output against the
    number after '####' in the reference answer."""
    decode = decode or (lambda t: bytes([x % 256 for x in t]).decode("utf-8", "replace"))
    correct = 0
    for r in rows:
        ids = _encode(model, "Question: " + r["question"] + "\nAnswer:")
        toks, _, _ = model.generate(ids, max_new_tokens)
        nums = _NUM.findall(decode(toks))
        gold = r["answer"].split("####")[-1].strip().replace(",", "")
        correct += int(bool(nums) and nums[-1].replace(",", "").rstrip(".") == gold)
    return Result("gsm8k", model.name, model.device, dict(n=len(rows), accuracy=correct / max(1, len(rows))))


def perplexity(model, ids: list[int], window: int = 512) -> Result:
    r = E.perplexity(model.logits, ids, window=window, stride=window // 2)
    return Result("ppl", model.name, model.device, dict(tokens=r.tokens, nll=r.nll, ppl=r.ppl))


def save_reference(model, prompts: list[list[int]], path: str):
    torch.save({"prompts": prompts, "logits": [model.logits(p)[-1].float().cpu() for p in prompts]}, path)


def parity(model, ref: str | object, prompts: list[list[int]] | None = None) -> Result:
    """Against a dump written by ``save_reference`` or another adapter."""
    if isinstance(ref, str):
        d = torch.load(ref)
        prompts, refs = d["prompts"], d["logits"]
    else:
        refs = [ref.logits(p)[-1].float().cpu() for p in prompts]
    match, cos = 0, []
    for p, r in zip(prompts, refs):
        lg = model.logits(p)[-1].float().cpu()
        match += int(int(lg.argmax()) == int(r.argmax()))
        cos.append(float(torch.nn.functional.cosine_similarity(lg, r, dim=0)))
    return Result("parity", model.name, model.device, dict(
        prompts=len(prompts), argmax_match=match == len(prompts), argmax_agree=match / max(1, len(prompts)),
        cosine_min=min(cos) if cos else math.nan, cosine_mean=sum(cos) / max(1, len(cos))))


def report(results: list[Result], path: str):
    with open(path, "w") as f:
        f.write("| model | device | kind | metrics |\n|---|---|---|---|\n")
        for r in results:
            f.write(r.row() + "\n")


# ---------------------------------------------------------------------------
# CLI
# ---------------------------------------------------------------------------

def build(args):
    if args.dry_run:
        return MockModel()
    from ..api import load
    return EngineModel(load(args.model), args.model)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("task", choices=["speed", "mc", "gsm8k", "ppl", "parity", "all"])
    ap.add_argument("--model", default="qwen3-0.6b")
    ap.add_argument("--dry-run", action="store_true")
    ap.add_argument("--data", default=None)
    ap.add_argument("--limit", type=int, default=None)
    ap.add_argument("--mode", default="letter", choices=["letter", "raw"])
    ap.add_argument("--text", default=None)
    ap.add_argument("--ref", default=None)
    ap.add_argument("--save-ref", default=None)
    ap.add_argument("--prompt-len", type=int, default=128)
    ap.add_argument("--gen-len", type=int, default=64)
    ap.add_argument("--report", default=None)
    a = ap.parse_args(argv)
    m = build(a)
    out = []
    if a.task in ("speed", "all"):
        out.append(speed(m, a.prompt_len, a.gen_len))
    if a.task in ("mc", "all"):
        rows = load_jsonl(a.data, a.limit) if a.data else synthetic_mc()
        if not a.data:
            print("warning: no --data; using the built-in synthetic multiple-choice set")
        out.append(multiple_choice(m, rows, a.mode))
    if a.task == "gsm8k":
        out.append(gsm8k(m, load_jsonl(a.data, a.limit)))
    if a.task in ("ppl", "all"):
        ids = _encode(m, open(a.text).read()) if a.text else [2 + i % 200 for i in range(300)]
        out.append(perplexity(m, ids))
    if a.task in ("parity", "all"):
        prompts = [list(range(3 + i, 40 + i)) for i in range(4)]
        if a.save_ref:
            save_reference(m, prompts, a.save_ref)
        if a.ref:
            out.append(parity(m, a.ref))
    for r in out:
        print(r.line(), flush=True)
    if a.report:
        report(out, a.report)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
