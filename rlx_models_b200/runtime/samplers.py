"""Logit processors for the less common samplers, applied per row to the
fp32 logits of a step before the GPU sampling kernel (temperature, top-k,
top-p, min-p and the draw itself stay in that kernel).

* typical (locally typical sampling, Meister et al. 2022): keep the tokens
  whose surprise -log p is closest to the entropy, smallest set with mass >=
  ``typical_p``;
* XTC (exclude top choices): with probability ``xtc_probability``, drop every
  token with p >= ``xtc_threshold`` except the least likely of them, when at
  least two qualify;
* DRY (don't repeat yourself): a token that would extend a repetition of
  length L >= ``dry_allowed_length`` of an earlier part of the context is
  penalised by ``dry_multiplier * dry_base ** (L - dry_allowed_length)``;
* Mirostat v2 (Basu et al. 2021): truncate tokens whose surprise in bits
  exceeds the running target mu, then mu -= eta * (surprise of the drawn token
  - tau); mu starts at 2 tau and lives with the request.

Order of application: penalties (kernel), DRY, typical, XTC, Mirostat; the
sampling kernel then applies temperature / top-k / top-p / min-p.

Reference: the host sampler of crates/rlx-qwen3/src/sampling.rs:41-400
(typical, XTC, DRY, mirostat among its modes).
"""
from __future__ import annotations

import math
import random

import torch


def typical_mask(x: torch.Tensor, p: float) -> torch.Tensor:
    lp = torch.log_softmax(x.float(), -1)
    prob = lp.exp()
    ent = -(prob * lp).nan_to_num().sum()
    score = (-lp - ent).abs()
    order = torch.argsort(score)
    cum = prob[order].cumsum(0)
    keep_n = int((cum < p).sum()) + 1
    out = torch.full_like(x, float("-inf"))
    idx = order[:keep_n]
    out[idx] = x[idx]
    return out


def xtc(x: torch.Tensor, threshold: float, probability: float, rng: random.Random) -> torch.Tensor:
    if probability <= 0 or rng.random() >= probability:
        return x
    prob = torch.softmax(x.float(), -1)
    top = (prob >= threshold).nonzero().flatten()
    if top.numel() < 2:
        return x
    keep = top[prob[top].argmin()]
    out = x.clone()
    drop = top[top != keep]
    out[drop] = float("-inf")
    return out


def dry_penalties(context: list[int], multiplier: float, base: float, allowed: int, last_n: int = -1,
                  breakers: set | None = None) -> dict[int, float]:
    """token -> penalty for extending a repeated suffix of ``context``."""
    if multiplier <= 0 or len(context) < 2:
        return {}
    ctx = context if last_n is None or last_n < 0 else context[-last_n:]
    n = len(ctx)
    breakers = breakers or set()
    best: dict[int, int] = {}
    last = ctx[-1]
    for j in range(n - 2, -1, -1):  # earlier occurrences of the last token
        if ctx[j] != last or ctx[j] in breakers:
            continue
        L = 1
        while L <= j and ctx[j - L] == ctx[n - 1 - L] and ctx[j - L] not in breakers:
            L += 1
        nxt = ctx[j + 1]
        if L >= allowed and nxt not in breakers:
            best[nxt] = max(best.get(nxt, 0), L)
    return {t: multiplier * base ** (L - allowed) for t, L in best.items()}


def mirostat_v2(x: torch.Tensor, mu: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Truncated logits and the untruncated log2-probabilities (for the update)."""
    lp2 = torch.log_softmax(x.float(), -1) / math.log(2.0)
    out = x.clone()
    surprise = -lp2
    cut = surprise > mu
    if bool(cut.all()):  # always keep the most likely token
        cut[int(lp2.argmax())] = False
    out[cut] = float("-inf")
    return out, lp2


def needs_processing(p) -> bool:
    return (getattr(p, "typical_p", 1.0) < 1.0 or getattr(p, "xtc_probability", 0.0) > 0
            or getattr(p, "dry_multiplier", 0.0) > 0 or getattr(p, "mirostat", 0) == 2)


def process_row(x: torch.Tensor, p, state, context: list[int]) -> torch.Tensor:
    """Apply the configured processors to one row ``x`` [V] (in place where
    possible); ``state`` is the request's RequestState (mirostat mu, RNG)."""
    if p.dry_multiplier > 0:
        pen = dry_penalties(context, p.dry_multiplier, p.dry_base, p.dry_allowed_length, p.dry_penalty_last_n)
        if pen:
            idx = torch.tensor(list(pen), device=x.device)
            x[idx] -= torch.tensor(list(pen.values()), device=x.device, dtype=x.dtype)
    if p.typical_p < 1.0:
        x.copy_(typical_mask(x, p.typical_p))
    if p.xtc_probability > 0:
        if state.rng is None:
            state.rng = random.Random(p.seed * 7919 + state.seq_id)
        x.copy_(xtc(x, p.xtc_threshold, p.xtc_probability, state.rng))
    if p.mirostat == 2:
        if state.mirostat_mu is None:
            state.mirostat_mu = 2.0 * p.mirostat_tau
        y, lp2 = mirostat_v2(x / max(p.temperature, 1e-6) if p.temperature > 0 else x, state.mirostat_mu)
        state.mirostat_lp2 = lp2
        x.copy_(torch.where(torch.isinf(y), y, x))
    return x


def mirostat_update(p, state, token: int):
    if p.mirostat == 2 and state.mirostat_lp2 is not None:
        s = -float(state.mirostat_lp2[token])
        state.mirostat_mu -= p.mirostat_eta * (s - p.mirostat_tau)
        state.mirostat_lp2 = None
