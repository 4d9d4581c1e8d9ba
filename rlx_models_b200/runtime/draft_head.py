"""Learned draft head for speculative decoding (EAGLE-style feature recurrence).

The head predicts the target's next tokens from the target's own features:

    x_t  = W_in [embed(token_{t+1}); h_t]            (2H -> H)
    y    = one causal transformer layer over x        (RMSNorm, MHA, SwiGLU)
    p    = softmax(lm_head(rmsnorm(y_t)))             -> token_{t+2}

``h_t`` is the target's final-normed hidden state at position t (the feature
its LM head turns into token t+1); the token embedding and the LM head are
the target's own (shared, frozen). Drafting k tokens recurs on the head's own
output features: after the first step, y_t stands in for the target feature.

Training is self-distillation: run the target over token sequences, take its
hidden states and next-token distributions, and minimise the KL divergence of
the head's prediction at t to the target's distribution at t + 1 (teacher
forcing on the target's features). Everything here is small (one layer of the
target's width) and runs in torch next to the target.

Reference: crates/rlx-eagle3 (EAGLE-3 draft heads), crates/rlx-dflash; the
draft / verify loop of crates/rlx-qwen3/src/spec.rs.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


class DraftHead(torch.nn.Module):
    def __init__(self, hidden: int, embed: torch.Tensor, lm_head: torch.Tensor, heads: int = 4,
                 mlp_mult: int = 2, eps: float = 1e-6):
        super().__init__()
        H = hidden
        self.H, self.nh, self.eps = H, heads, eps
        self.register_buffer("embed", embed.detach().float(), persistent=False)
        self.register_buffer("lm_head", lm_head.detach().float(), persistent=False)
        g = torch.Generator().manual_seed(0)
        init = lambda *s: torch.nn.Parameter(torch.randn(*s, generator=g) / math.sqrt(s[-1]))  # noqa: E731
        self.w_in = init(H, 2 * H)
        self.ln1 = torch.nn.Parameter(torch.ones(H))
        self.wqkv = init(3 * H, H)
        self.wo = torch.nn.Parameter(torch.zeros(H, H))
        self.ln2 = torch.nn.Parameter(torch.ones(H))
        self.w_gu = init(2 * mlp_mult * H, H)
        self.w_dn = torch.nn.Parameter(torch.zeros(H, mlp_mult * H))
        self.ln_out = torch.nn.Parameter(torch.ones(H))

    def _norm(self, x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * w

    def features(self, h: torch.Tensor, next_tokens: torch.Tensor) -> torch.Tensor:
        """h [B, T, H] target (or draft) features, next_tokens [B, T] -> y [B, T, H]."""
        x = torch.cat([self.embed[next_tokens], h.float()], -1) @ self.w_in.t()
        B, T, H = x.shape
        a = self._norm(x, self.ln1) @ self.wqkv.t()
        q, k, v = (t.view(B, T, self.nh, H // self.nh).transpose(1, 2) for t in a.split(H, -1))
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B, T, H)
        x = x + o @ self.wo.t()
        g, u = (self._norm(x, self.ln2) @ self.w_gu.t()).chunk(2, -1)
        return x + (F.silu(g) * u) @ self.w_dn.t()

    def logits(self, y: torch.Tensor) -> torch.Tensor:
        return self._norm(y, self.ln_out) @ self.lm_head.t()

    @torch.no_grad()
    def propose(self, h_ctx: torch.Tensor, tok_ctx: list[int], k: int) -> list[int]:
        """``h_ctx`` [W, H]: target features of the last W positions; ``tok_ctx``:
        the W tokens that followed them (the last is the newest token). Returns
        k greedy draft tokens."""
        dev = self.w_in.device
        h = h_ctx.float().to(dev).unsqueeze(0)
        toks = torch.tensor([tok_ctx], device=dev)
        out = []
        for _ in range(k):
            y = self.features(h, toks)
            nxt = int(self.logits(y[:, -1]).argmax(-1))
            out.append(nxt)
            h = torch.cat([h, y[:, -1:]], 1)  # the head's own feature stands in for the target's
            toks = torch.cat([toks, torch.tensor([[nxt]], device=dev)], 1)
        return out


def distill_step(head: DraftHead, opt, h: torch.Tensor, tokens: torch.Tensor, target_logits: torch.Tensor) -> float:
    """One optimisation step. h [B, T, H] target features at positions 0..T-1,
    tokens [B, T + 1], target_logits [B, T, V] (position t predicts token t+1).
    The head at t sees (h_t, token_{t+1}) and matches the target at t + 1."""
    y = head.features(h[:, :-1], tokens[:, 1:-1])
    lp = torch.log_softmax(head.logits(y), -1)
    tp = torch.softmax(target_logits[:, 1:].float(), -1)
    loss = F.kl_div(lp, tp, reduction="batchmean") / y.shape[1]
    opt.zero_grad()
    loss.backward()
    opt.step()
    return float(loss.detach())


def train_draft_head(head: DraftHead, target_fn, sequences: list[list[int]], steps: int = 200, lr: float = 3e-3,
                     window: int = 64) -> list[float]:
    """``target_fn(ids) -> (hidden [T, H], logits [T, V])`` of the target over
    a token list (e.g. the fp32 oracle or the GPU model through a helper)."""
    opt = torch.optim.Adam([p for p in head.parameters() if p.requires_grad], lr=lr)
    data = []
    with torch.no_grad():
        for s in sequences:
            hs, lg = target_fn(s)
            data.append((hs.float(), torch.tensor(s), lg.float()))
    losses = []
    dev = head.w_in.device
    for it in range(steps):
        hs, toks, lg = data[it % len(data)]
        n = hs.shape[0]
        a = (it * 7919) % max(1, n - 1 - window) if n - 1 > window else 0
        b = min(n - 1, a + window)  # features a..b-1 need tokens a..b
        losses.append(distill_step(head, opt, hs[a:b].unsqueeze(0).to(dev), toks[a:b + 1].unsqueeze(0).to(dev),
                                   lg[a:b].unsqueeze(0).to(dev)))
    return losses
