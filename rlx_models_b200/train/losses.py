"""Preference-optimisation losses on top of the trainable decoder.

``sequence_logprob`` sums log p(target) over each row's unmasked targets
(one fused lm_head + CE pass per row); ``dpo_loss`` is the DPO objective
-log sigmoid(beta * ((pi_c - ref_c) - (pi_r - ref_r))).

Reference: rlx-tune src/loss.rs (DPO), src/dpo*.rs.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def sequence_logprob(model, ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """[B] summed target log-probabilities (differentiable)."""
    out = []
    for b in range(ids.shape[0]):
        # model.loss with denom 1 is the summed CE = -sum log p
        out.append(-model.loss(ids[b:b + 1], targets[b:b + 1], denom=1.0))
    return torch.stack(out)


def dpo_loss(pi_chosen, pi_rejected, ref_chosen, ref_rejected, beta: float = 0.1) -> torch.Tensor:
    margin = beta * ((pi_chosen - ref_chosen) - (pi_rejected - ref_rejected))
    return -F.logsigmoid(margin).mean()
