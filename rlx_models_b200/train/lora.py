"""LoRA / DoRA adapters for the trainable decoder.

Per transformer layer and target linear (``qkv``, ``o``, ``gate_up``,
``down``): A [r, in] ~ N(0, 1/r), B [out, r] = 0, scale alpha / r, so
``y = x W^T + s (x A^T) B^T``. DoRA (weight-decomposed LoRA) adds a learned
magnitude m [out] initialised to the row norms of W and uses
``W' = m * V / ||V||_row`` with ``V = W + s B A`` (the norm is detached, as
in the DoRA paper's memory-efficient form). Base weights are frozen (their
FSDP groups are gathered without autograd, so no weight gradients or
reduce-scatters run); adapters are small and replicated on every rank as one
flat group whose gradient is all-reduced (data parallel). ``merged()`` folds
the adapters into HF-named base weights for export.

Reference: rlx-tune src/adapter.rs, src/inject.rs (LoRA / DoRA injection,
fuse for export).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import functional as TF
from .fsdp import FlatGroup, gather_params

TARGETS = ("qkv", "o", "gate_up", "down")


def _dims(cfg, t):
    H, I = cfg.hidden_size, cfg.intermediate_size
    return {"qkv": (cfg.q_size + 2 * cfg.kv_size, H), "o": (H, cfg.q_size), "gate_up": (2 * I, H),
            "down": (H, I)}[t]


class LoraAdapters:
    def __init__(self, model, r: int = 16, alpha: float = 32.0, targets=TARGETS, dora: bool = False, seed: int = 0,
                 group=None, world: int = 1):
        cfg = model.cfg
        self.model, self.r, self.scale, self.dora = model, r, alpha / r, dora
        self.targets = tuple(targets)
        self.world, self.group = world, group
        g = torch.Generator().manual_seed(seed)
        named = []
        for i in range(cfg.num_hidden_layers):
            base = None
            if dora:
                with torch.no_grad():
                    base = dict(zip(self._layer_names(cfg), gather_params(model.layers[i])))
            for t in self.targets:
                out, inp = _dims(cfg, t)
                named.append((f"{i}.{t}.A", torch.randn(r, inp, generator=g) / math.sqrt(r)))
                named.append((f"{i}.{t}.B", torch.zeros(out, r)))
                if dora:
                    named.append((f"{i}.{t}.m", base[t].float().norm(dim=1).cpu()))
        # replicated (world 1) flat group: the trainer all-reduces its gradient
        self.group_flat = FlatGroup("lora", named, 0, 1, model.device, None, torch.bfloat16)
        self.index = {n: k for k, (n, _) in enumerate(named)}
        for fg in model.groups:
            fg.frozen = True

    @staticmethod
    def _layer_names(cfg):
        return (["ln1", "qkv"] + (["qn", "kn"] if cfg.qk_norm else []) + ["o", "ln2", "gate_up", "down"])

    def params(self) -> list[torch.Tensor]:
        return gather_params(self.group_flat)

    def linear(self, params, i: int, t: str, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        if t not in self.targets:
            return TF.linear(x, w)
        A = params[self.index[f"{i}.{t}.A"]]
        B = params[self.index[f"{i}.{t}.B"]]
        y = TF.linear(x, w) + self.scale * TF.linear(TF.linear(x, A), B)
        if self.dora:
            m = params[self.index[f"{i}.{t}.m"]]
            with torch.no_grad():
                V = w.float() + self.scale * (B.float() @ A.float())
                norm = V.norm(dim=1).clamp_min(1e-12)
            y = y * (m.float() / norm).to(y.dtype)
        return y

    def allreduce_grad(self):
        if self.world > 1:
            dist.all_reduce(self.group_flat.grad, group=self.group)
            self.group_flat.grad /= self.world

    @torch.no_grad()
    def merged(self) -> dict[str, torch.Tensor]:
        """HF-named fused weights with the adapters folded in (fp32)."""
        cfg, params = self.model.cfg, self.params()
        out = {}
        for i in range(cfg.num_hidden_layers):
            named = dict(zip(self._layer_names(cfg), gather_params(self.model.layers[i])))
            for t in self.targets:
                A = params[self.index[f"{i}.{t}.A"]].float()
                B = params[self.index[f"{i}.{t}.B"]].float()
                W = named[t].float() + self.scale * (B @ A)
                if self.dora:
                    m = params[self.index[f"{i}.{t}.m"]].float()
                    W = W * (m / W.norm(dim=1).clamp_min(1e-12))[:, None]
                out[(i, t)] = W
        return out
