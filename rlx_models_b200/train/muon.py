"""Muon: orthogonalized momentum for 2-D weight matrices (AdamW for the rest).

Update of one weight matrix W with gradient G (after clipping):

    M  = mu * M + G                        momentum
    N  = G + mu * M                        Nesterov look-ahead
    O  = NewtonSchulz5(N)                  approximately the orthogonal factor U V^T of N
    W -= lr * (sqrt(max(1, rows / cols)) * O + wd * W)

NewtonSchulz5 is the quintic iteration X <- a X + (b A + c A^2) X with
A = X X^T on X = N / ||N||_F (transposed so that rows <= cols), with the
coefficients (a, b, c) = (3.4445, -4.7750, 2.0315) and 5 steps published with
the method (K. Jordan et al., "Muon: An optimizer for hidden layers in neural
networks", 2024); it runs in bf16 like the published version. One-dimensional
parameters (norm weights) and embeddings keep AdamW.

The reference's Muon group is single-process only because it needs whole
matrices (rlx-tune src/trainer.rs:386-433, :920). Here the momentum stays
sharded like the other optimizer state: each rank updates its shard of M,
all-gathers the group's Nesterov direction N, orthogonalizes every 2-D
parameter (identically on every rank) and applies its own slice of the
update, so Muon also works under FSDP.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

NS_COEFFS = (3.4445, -4.7750, 2.0315)


def newton_schulz5(g: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    a, b, c = NS_COEFFS
    x = g.to(torch.bfloat16 if g.is_cuda else torch.float32)
    tr = x.shape[0] > x.shape[1]
    if tr:
        x = x.t()
    x = x / (x.float().norm() + eps).to(x.dtype)
    for _ in range(steps):
        A = x @ x.t()
        B = b * A + c * (A @ A)
        x = a * x + B @ x
    if tr:
        x = x.t()
    return x.float()


def muon_step(trainer, g, lr: float, skip_names=("embed_tokens", "lm_head")):
    """One Muon + AdamW update of the FlatGroup ``g`` (see module docstring).
    ``trainer`` supplies the config (betas, eps, weight decay, momentum), the
    step number and the clip coefficient."""
    c = trainer.cfg
    mu = c.muon_momentum
    coef = trainer._coef if torch.is_tensor(trainer._coef) else float(trainer._coef)
    gr = g.grad * coef
    if getattr(g, "muon_buf", None) is None:
        g.muon_buf = torch.zeros_like(g.master)
    g.muon_buf.mul_(mu).add_(gr)
    nes = gr + mu * g.muon_buf
    # AdamW direction for every element (1-D parameters keep it)
    b1, b2 = c.betas
    g.exp_avg.mul_(b1).add_(gr, alpha=1 - b1)
    g.exp_avg_sq.mul_(b2).addcmul_(gr, gr, value=1 - b2)
    step = trainer.step_num
    upd = (g.exp_avg / (1 - b1 ** step)) / ((g.exp_avg_sq / (1 - b2 ** step)).sqrt() + c.eps)
    # Muon direction for the 2-D matrices, from the all-gathered Nesterov momentum
    if g.world > 1:
        if g.device.type == "cpu":
            parts = [torch.empty_like(nes) for _ in range(g.world)]
            dist.all_gather(parts, nes, group=g.group)
            full = torch.cat(parts)
        else:
            full = torch.empty(g.padded, dtype=nes.dtype, device=nes.device)
            dist.all_gather_into_tensor(full, nes, group=g.group)
    else:
        full = nes
    lo, hi = g.rank * g.shard_n, (g.rank + 1) * g.shard_n
    for name, off, n, shape in zip(g.names, g.offsets, g.numels, g.shapes):
        if len(shape) != 2 or min(shape) < 2 or any(s in name for s in skip_names):
            continue
        a, b = max(lo, off), min(hi, off + n)
        if a >= b:
            continue
        o = newton_schulz5(full[off:off + n].view(shape)) * max(1.0, shape[0] / shape[1]) ** 0.5
        upd[a - lo:b - lo] = o.reshape(-1)[a - off:b - off]
    g.master.mul_(1 - lr * c.weight_decay).sub_(lr * upd)
    g.param.copy_(g.master)
