"""Speculative decoding: draft, then verify k tokens in one target pass.

Greedy draft-and-verify: a proposer suggests ``k`` tokens after the last
accepted one; the target runs the last accepted token plus the ``k``
proposals as one causal chunk (k + 1 positions, logits at every position),
accepts the longest prefix that equals its own argmax and appends its own
token at the first disagreement (or a bonus token when all k match). The
output is the target's greedy continuation; each target pass yields between
1 and k + 1 tokens.

Proposers:
  * a draft model (any decoder with the same vocabulary) decoding greedily on
    its own paged KV cache, rolled back by position after each verification;
  * prompt lookup (no model): the tokens that followed the most recent earlier
    occurrence of the current n-gram suffix (n = ngram .. 1).

KV caches are positional (slot = position under an identity block table), so
rolling back after a rejection is just moving the position: stale entries past
it are overwritten by the next writes.

  * a learned draft head (runtime/draft_head.py): the target's own final
    features plus the newest token through one small layer, recurring on its
    own features for the following drafts.

Reference: rlx-qwen3 src/spec.rs (draft / verify loop), rlx-eagle3 and
rlx-dflash (learned draft heads).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.decoder import ForwardBatch


@dataclass
class SpecStats:
    target_passes: int = 0
    proposed: int = 0
    accepted: int = 0

    @property
    def acceptance(self) -> float:
        return self.accepted / max(1, self.proposed)

    @property
    def tokens_per_pass(self) -> float:
        return (self.accepted + self.target_passes) / max(1, self.target_passes)


class _Seq:
    """A model plus its own paged cache for one sequence (identity block table)."""

    def __init__(self, model, max_len: int):
        self.model = model
        self.nb = (max_len + 15) // 16 + 1
        self.kv = model.make_kv_cache(self.nb)
        dev = model.device
        self.table = torch.arange(self.nb, dtype=torch.int32, device=dev).view(1, -1)
        self.pos = 0  # positions [0, pos) hold valid K/V
        self.hidden = None  # [max_len, H] final-normed features per position (draft-head proposers)

    @torch.no_grad()
    def run(self, tokens: list[int], start: int, keep_hidden: bool = False) -> torch.Tensor:
        """Feed ``tokens`` at positions start.. ; returns fp32 logits per token [n, V]."""
        dev = self.model.device
        n = len(tokens)
        ctx = start + n
        if ctx > self.nb * 16:
            raise ValueError("sequence longer than the speculative decoder's max_len")
        fb = ForwardBatch(input_ids=torch.tensor(tokens, dtype=torch.int32, device=dev),
                          positions=torch.arange(start, ctx, dtype=torch.int32, device=dev),
                          slots=torch.arange(start, ctx, dtype=torch.int64, device=dev), num_decode=0,
                          pre_block_tables=self.table, pre_ctx_lens=torch.tensor([ctx], dtype=torch.int32, device=dev),
                          pre_cu_q=torch.tensor([0, n], dtype=torch.int32, device=dev), pre_max_q=n)
        if keep_hidden:
            h = self.model.forward_hidden(fb, self.kv)
            if self.hidden is None:
                self.hidden = torch.zeros(self.nb * 16, h.shape[1], dtype=h.dtype, device=dev)
            self.hidden[start:ctx] = h
            out = self.model.logits(h)
        else:
            out = self.model.forward(fb, self.kv)
        self.pos = ctx
        return out


_STATE_ATTRS = ("conv", "rec", "ssm")  # per-slot recurrent state tensors [layers, slots, ...] of hybrid caches


def _snapshot(kv, slot: int = 0) -> dict:
    return {a: getattr(kv, a)[:, slot].clone() for a in _STATE_ATTRS if hasattr(kv, a)}


def _restore(kv, snap: dict, slot: int = 0) -> None:
    for a, t in snap.items():
        getattr(kv, a)[:, slot].copy_(t)


class SpeculativeDecoder:
    def __init__(self, target, draft=None, k: int = 4, max_len: int = 4096, ngram: int = 3, draft_head=None,
                 head_window: int = 16):
        if draft is not None and getattr(draft, "stateful", False) and draft is not target:
            raise NotImplementedError("a recurrent-state draft model cannot roll back rejected tokens")
        # recurrent-state targets (linear attention / SSM layers): the verify pass advances the
        # state over every proposal, so a partial acceptance restores the state saved before it
        # and re-runs the accepted tokens (attention KV rolls back by position as before)
        self.stateful = bool(getattr(target, "stateful", False))
        self.target = _Seq(target, max_len)
        self.draft = _Seq(draft, max_len) if draft is not None else None
        self.head, self.head_window = draft_head, head_window
        self.k, self.ngram = k, ngram
        self.stats = SpecStats()

    def _propose_head(self, seq: list[int], k: int) -> list[int]:
        """Learned draft head over the target's features of the last positions."""
        last = len(seq) - 2  # feature that produced the newest token
        a = max(0, last - self.head_window + 1)
        kw = {"pos0": a + 1} if getattr(self.head, "uses_positions", False) else {}  # RoPE'd heads (MTP)
        return self.head.propose(self.target.hidden[a:last + 1], seq[a + 1:last + 2], k, **kw)

    # -- proposers ---------------------------------------------------------------
    def _propose_draft(self, seq: list[int], k: int) -> list[int]:
        d = self.draft
        # catch up: feed every accepted token the draft has not seen (the last one included)
        pending = seq[d.pos:]
        lg = d.run(pending, d.pos)
        props = [int(lg[-1].argmax())]
        for _ in range(k - 1):
            lg = d.run([props[-1]], d.pos)
            props.append(int(lg[-1].argmax()))
        return props

    def _propose_lookup(self, seq: list[int], k: int) -> list[int]:
        for n in range(min(self.ngram, len(seq) - 1), 0, -1):
            suf = seq[-n:]
            for s in range(len(seq) - n - 1, -1, -1):
                if seq[s:s + n] == suf:
                    nxt = seq[s + n:s + n + k]
                    if nxt:
                        return nxt
        return []

    # -- generation --------------------------------------------------------------
    @torch.no_grad()
    def generate(self, prompt: list[int], max_new_tokens: int, eos_token_id: int | None = None) -> list[int]:
        t = self.target
        t.pos = 0
        if self.draft is not None:
            self.draft.pos = 0
        keep = self.head is not None
        lg = t.run(list(prompt), 0, keep)
        seq = list(prompt) + [int(lg[-1].argmax())]
        out = [seq[-1]]
        while len(out) < max_new_tokens and (eos_token_id is None or out[-1] != eos_token_id):
            k = min(self.k, max_new_tokens - len(out))
            if self.head is not None:
                props = self._propose_head(seq, k)
            elif self.draft is not None:
                props = self._propose_draft(seq, k)
            else:
                props = self._propose_lookup(seq, k)
            # verify: the last accepted token (not yet in the target cache) + proposals
            start = len(seq) - 1
            snap = _snapshot(t.kv) if self.stateful and props else None
            lv = t.run([seq[-1]] + props, start, keep)
            tgt = lv.argmax(-1).tolist()
            n_acc = 0
            while n_acc < len(props) and props[n_acc] == tgt[n_acc]:
                n_acc += 1
            if snap is not None and n_acc < len(props):
                _restore(t.kv, snap)
                t.run([seq[-1]] + props[:n_acc], start, keep)
            new = props[:n_acc] + [tgt[n_acc]]
            self.stats.target_passes += 1
            self.stats.proposed += len(props)
            self.stats.accepted += n_acc
            if eos_token_id is not None and eos_token_id in new:
                new = new[:new.index(eos_token_id) + 1]
            new = new[:max_new_tokens - len(out)]
            seq += new
            out += new
            t.pos = len(seq) - 1  # the newest token is not in the cache yet
            if self.draft is not None:
                self.draft.pos = min(self.draft.pos, len(seq) - 1)
        return out
