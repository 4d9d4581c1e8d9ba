"""Fully sharded data parallel (ZeRO-3) parameter groups.

Each group (one transformer layer, or the embedding/norm/head set) keeps its
parameters as one flat buffer, sharded over the data-parallel ranks:

* bf16 parameter shard (what the all-gather sends),
* fp32 master shard + AdamW moments (updated in place by the fused AdamW kernel,
  which also writes the bf16 shard, so the cast is fused into the update),
* fp32 gradient shard accumulator.

``GatherParams`` is the autograd boundary: forward all-gathers the shards and
returns the full weights as views; backward concatenates their gradients and
reduce-scatters them (sum) into the gradient shard. With per-layer activation
checkpointing the gather runs again in the recompute, so only one layer's
full parameters are live at a time.

The reference has no parameter sharding; its closest mode is ZeRO-1
(rlx-tune src/trainer.rs:1055-1082: reduce_scatter_mean -> clip -> shard step ->
all_gather_into), which this generalises to sharded parameters as well.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


class FlatGroup:
    ALIGN = 128  # elements; keeps every shard 16-byte aligned

    def __init__(self, name: str, named: list[tuple[str, torch.Tensor]], rank: int, world: int, device,
                 group=None, param_dtype: torch.dtype = torch.bfloat16):
        self.name = name
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device(device)
        self.names = [n for n, _ in named]
        self.shapes = [tuple(t.shape) for _, t in named]
        self.numels = [t.numel() for _, t in named]
        self.offsets = []
        off = 0
        for n in self.numels:
            self.offsets.append(off)
            off += n
        self.numel = off
        unit = self.ALIGN * world
        self.padded = math.ceil(off / unit) * unit
        self.shard_n = self.padded // world
        lo, hi = rank * self.shard_n, (rank + 1) * self.shard_n
        master = torch.zeros(self.shard_n, dtype=torch.float32, device=self.device)
        # copy only the slice of each tensor that falls in this rank's shard
        for (_, t), o, n in zip(named, self.offsets, self.numels):
            a, b = max(lo, o), min(hi, o + n)
            if a < b:
                master[a - lo:b - lo] = t.reshape(-1)[a - o:b - o].to(self.device, torch.float32)
        self.master = master
        self.param = master.to(param_dtype)
        self.exp_avg = torch.zeros_like(master)
        self.exp_avg_sq = torch.zeros_like(master)
        self.grad = torch.zeros_like(master)
        self.anchor = torch.zeros((), device=self.device, requires_grad=True)  # autograd hook for backward
        self.frozen = False  # frozen groups are gathered without autograd (no weight gradients)

    # -- collective helpers ---------------------------------------------------
    def _gloo(self) -> bool:
        return self.device.type == "cpu"

    def all_gather(self) -> torch.Tensor:
        if self.world == 1:
            return self.param
        if self._gloo():  # CPU test path (gloo has no *_into_tensor collectives)
            parts = [torch.empty_like(self.param) for _ in range(self.world)]
            dist.all_gather(parts, self.param, group=self.group)
            return torch.cat(parts)
        full = torch.empty(self.padded, dtype=self.param.dtype, device=self.device)
        dist.all_gather_into_tensor(full, self.param, group=self.group)
        return full

    def reduce_scatter_add(self, full_grad: torch.Tensor):
        if self.world == 1:
            self.grad += full_grad[:self.shard_n]
            return
        if self._gloo():
            dist.all_reduce(full_grad, group=self.group)
            self.grad += full_grad[self.rank * self.shard_n:(self.rank + 1) * self.shard_n]
            return
        out = torch.empty(self.shard_n, dtype=full_grad.dtype, device=self.device)
        dist.reduce_scatter_tensor(out, full_grad, op=dist.ReduceOp.SUM, group=self.group)
        self.grad += out

    def views(self, flat: torch.Tensor) -> list[torch.Tensor]:
        return [flat[o:o + n].view(s) for o, n, s in zip(self.offsets, self.numels, self.shapes)]

    def full_fp32(self) -> torch.Tensor:
        """Gather the fp32 master (checkpoint export)."""
        if self.world == 1:
            return self.master[:self.numel]
        if self._gloo():
            parts = [torch.empty_like(self.master) for _ in range(self.world)]
            dist.all_gather(parts, self.master, group=self.group)
            return torch.cat(parts)[:self.numel]
        full = torch.empty(self.padded, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(full, self.master, group=self.group)
        return full[:self.numel]

    def named_full(self) -> dict[str, torch.Tensor]:
        full = self.full_fp32()
        return {n: full[o:o + k].view(s) for n, o, k, s in zip(self.names, self.offsets, self.numels, self.shapes)}


class GatherParams(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, fg: FlatGroup):
        ctx.fg = fg
        full = fg.all_gather()
        return tuple(fg.views(full))

    @staticmethod
    def backward(ctx, *grads):
        fg: FlatGroup = ctx.fg
        flat = torch.zeros(fg.padded, dtype=torch.float32, device=fg.device)
        for g, o, n in zip(grads, fg.offsets, fg.numels):
            if g is not None:
                flat[o:o + n] = g.reshape(-1)
        fg.reduce_scatter_add(flat)
        return None, None


def gather_params(fg: FlatGroup) -> list[torch.Tensor]:
    if fg.frozen:
        with torch.no_grad():
            return list(fg.views(fg.all_gather()))
    return list(GatherParams.apply(fg.anchor, fg))
