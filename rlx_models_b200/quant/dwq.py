"""DWQ, distilled weight quantisation ("heal via adapter"): quantise a linear
layer's weight, freeze it, and train a low-rank adapter A·B on calibration
activations so that x·(W_q + A·B)ᵀ matches the full-precision x·Wᵀ. The
healed weight W_q + A·B runs as a dense layer (or is re-quantised); its output
error is far below the quantised layer's alone.

Quantisation-aware training (QAT) lives in the trainer (``TrainConfig.qat``):
the forward pass sees fake-quantised weights and gradients pass straight
through the rounding.

Reference: crates/rlx-tune/src/dwq.rs (`DwqResult`: healed weight, quant
error, DWQ error), trainer.rs:456-561 (`qat` number format).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .calib import FORMATS


class FakeQuant(torch.autograd.Function):
    """Forward: the weight rounded to ``fmt`` (quantise -> dequantise);
    backward: the identity (straight-through estimator)."""

    @staticmethod
    def forward(ctx, w, fmt: str):
        return FORMATS[fmt](w.float()).to(w.dtype)

    @staticmethod
    def backward(ctx, g):
        return g, None


def fake_quant(w: torch.Tensor, fmt: str) -> torch.Tensor:
    return FakeQuant.apply(w, fmt)


@dataclass
class DwqResult:
    healed_weight: torch.Tensor  # [out, in] = W_q + A B
    quant_error: float           # relative output error of W_q alone
    dwq_error: float             # relative output error of the healed weight


def heal_linear(w: torch.Tensor, x: torch.Tensor, fmt: str = "int4", rank: int = 16, steps: int = 300,
                lr: float = 1e-2, seed: int = 0) -> DwqResult:
    """``w`` [out, in], calibration inputs ``x`` [n, in]."""
    w = w.float()
    x = x.float()
    wq = FORMATS[fmt](w)
    target = x @ w.t()
    g = torch.Generator(device="cpu").manual_seed(seed)
    out_f, in_f = w.shape
    a = (torch.randn(out_f, rank, generator=g) * 0.0).to(w.device).requires_grad_(True)  # zero: start at W_q
    b = (torch.randn(rank, in_f, generator=g) / in_f ** 0.5).to(w.device).requires_grad_(True)
    opt = torch.optim.Adam([a, b], lr=lr)
    scale = target.pow(2).mean().clamp_min(1e-12)
    for _ in range(steps):
        opt.zero_grad()
        y = x @ (wq + a @ b).t()
        loss = (y - target).pow(2).mean() / scale
        loss.backward()
        opt.step()
    with torch.no_grad():
        healed = wq + a @ b
        qe = float((x @ wq.t() - target).norm() / target.norm())
        de = float((x @ healed.t() - target).norm() / target.norm())
    return DwqResult(healed, qe, de)
