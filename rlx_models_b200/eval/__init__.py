"""Evaluation: perplexity, multiple-choice log-likelihood scoring, and the
machine-translation metrics BLEU and chrF.

Every model-facing function takes a ``logits_fn(ids: list[int]) -> [T, V]``
callable (next-token logits at every position) so the same code scores the
GPU engine (``LLM.logits``) and the fp32 CPU oracle.

Reference: crates/rlx-eval/src/perplexity.rs, src/multiple_choice.rs;
crates/rlx-mt-eval (BLEU / chrF).
"""
from __future__ import annotations

import math
from collections import Counter
from dataclasses import dataclass
from typing import Callable, Sequence

import torch

LogitsFn = Callable[[list], torch.Tensor]


def token_logprobs(logits_fn: LogitsFn, ids: Sequence[int]) -> torch.Tensor:
    """log p(ids[t] | ids[:t]) for t = 1 .. len(ids) - 1 (fp32, CPU)."""
    ids = list(ids)
    lg = logits_fn(ids).float().cpu()
    lp = torch.log_softmax(lg[:-1], -1)
    return lp.gather(1, torch.tensor(ids[1:]).view(-1, 1)).squeeze(1)


@dataclass
class PerplexityResult:
    nll: float          # mean negative log-likelihood per scored token
    ppl: float
    tokens: int


def perplexity(logits_fn: LogitsFn, ids: Sequence[int], window: int = 1024, stride: int | None = None) \
        -> PerplexityResult:
    """Sliding-window perplexity. Every token after the first is scored
    exactly once; a chunk of up to ``stride`` target tokens (at most
    ``window - 1``) is scored from one forward over the ``window`` tokens that
    end with it, so each target sees as much left context as the window allows."""
    ids = list(ids)
    n = len(ids)
    chunk = max(1, min(stride or window, window - 1))
    total, count = 0.0, 0
    s = 1
    while s < n:
        e = min(s + chunk, n)
        begin = max(0, e - window)
        lp = token_logprobs(logits_fn, ids[begin:e])  # predictions for ids[begin + 1 : e]
        new = lp[s - begin - 1:]
        total -= float(new.sum())
        count += new.numel()
        s = e
    nll = total / max(1, count)
    return PerplexityResult(nll, math.exp(nll), count)


@dataclass
class ChoiceScores:
    logprob: list[float]       # summed log-likelihood of each continuation
    logprob_norm: list[float]  # per-token (length-normalised)
    best: int                  # argmax of the summed score
    best_norm: int


def multiple_choice(logits_fn: LogitsFn, context: Sequence[int], choices: Sequence[Sequence[int]]) -> ChoiceScores:
    """Score each continuation by log p(choice | context)."""
    ctx = list(context)
    lps, norms = [], []
    for ch in choices:
        ch = list(ch)
        lp = token_logprobs(logits_fn, ctx + ch)[len(ctx) - 1:]
        s = float(lp.sum())
        lps.append(s)
        norms.append(s / max(1, len(ch)))
    return ChoiceScores(lps, norms, int(max(range(len(lps)), key=lps.__getitem__)),
                        int(max(range(len(norms)), key=norms.__getitem__)))


def accuracy(logits_fn: LogitsFn, items: Sequence[tuple], normalised: bool = False) -> float:
    """``items``: (context ids, [choice ids ...], gold index)."""
    ok = 0
    for ctx, choices, gold in items:
        sc = multiple_choice(logits_fn, ctx, choices)
        ok += int((sc.best_norm if normalised else sc.best) == gold)
    return ok / max(1, len(items))


# ---------------------------------------------------------------------------
# machine-translation metrics (corpus level)
# ---------------------------------------------------------------------------

def _ngrams(tokens: Sequence[str], n: int) -> Counter:
    return Counter(tuple(tokens[i:i + n]) for i in range(len(tokens) - n + 1))


def bleu(hypotheses: Sequence[str], references: Sequence[Sequence[str]] | Sequence[str], max_n: int = 4,
         smooth: bool = False) -> float:
    """Corpus BLEU (0-100) over whitespace tokens: clipped n-gram precisions
    for n = 1..max_n, geometric mean, brevity penalty against the closest
    reference length. ``references``: one string per hypothesis or a list of
    reference strings per hypothesis."""
    match = [0] * max_n
    total = [0] * max_n
    hyp_len = ref_len = 0
    for hyp, refs in zip(hypotheses, references):
        refs = [refs] if isinstance(refs, str) else list(refs)
        h = hyp.split()
        rs = [r.split() for r in refs]
        hyp_len += len(h)
        ref_len += min((abs(len(r) - len(h)), len(r)) for r in rs)[1]
        for n in range(1, max_n + 1):
            hc = _ngrams(h, n)
            mx = Counter()
            for r in rs:
                for g, c in _ngrams(r, n).items():
                    mx[g] = max(mx[g], c)
            match[n - 1] += sum(min(c, mx[g]) for g, c in hc.items())
            total[n - 1] += max(0, len(h) - n + 1)
    if hyp_len == 0:
        return 0.0
    logs = []
    for n in range(max_n):
        m, t = match[n], total[n]
        if smooth:
            m, t = m + 1, t + 1
        if m == 0 or t == 0:
            return 0.0
        logs.append(math.log(m / t))
    bp = 1.0 if hyp_len > ref_len else math.exp(1 - ref_len / hyp_len)
    return 100.0 * bp * math.exp(sum(logs) / max_n)


def chrf(hypotheses: Sequence[str], references: Sequence[str], n_char: int = 6, beta: float = 2.0) -> float:
    """Corpus chrF (0-100): character n-gram (n = 1..n_char, spaces removed)
    precision and recall averaged over n, combined as F-beta."""
    precs, recs = [], []
    for n in range(1, n_char + 1):
        m = hp = rp = 0
        for hyp, ref in zip(hypotheses, references):
            h = _ngrams(list(hyp.replace(" ", "")), n)
            r = _ngrams(list(ref.replace(" ", "")), n)
            m += sum(min(c, r[g]) for g, c in h.items())
            hp += sum(h.values())
            rp += sum(r.values())
        if hp > 0 and rp > 0:
            precs.append(m / hp)
            recs.append(m / rp)
    if not precs:
        return 0.0
    p, r = sum(precs) / len(precs), sum(recs) / len(recs)
    if p + r == 0:
        return 0.0
    b2 = beta * beta
    return 100.0 * (1 + b2) * p * r / (b2 * p + r)
