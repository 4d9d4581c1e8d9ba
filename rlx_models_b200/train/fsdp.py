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

Gradient reduce-scatter has two implementations. The NCCL one materialises
each group's full fp32 gradient and calls ``reduce_scatter_tensor``. The push
one (``GradPush``, CUDA) keeps every rank's gradient shards in a symmetric IPC
heap and ADDS each gradient element straight into its owner's shard over
NVLink: the wgrad GEMM's epilogue pushes weight gradients tile by tile during
the backward pass (no full weight gradient is ever stored), and a push kernel
handles the remaining dense gradients (norms, embedding / lm_head); one
device barrier before the optimizer makes every rank's pushes visible.

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
        self.push_table = None  # GradPush: int64 [world] device addresses of every rank's grad shard
        self.gathered = (0, 0)  # [start, end) byte range of the live gathered bf16 params
        self._prefetched = None  # (full params, event) of an all-gather started by prefetch()

    # -- collective helpers ---------------------------------------------------
    def _gloo(self) -> bool:
        return self.device.type == "cpu"

    def prefetch(self):
        """Start this group's parameter all-gather on the communication stream,
        so it overlaps the compute queued after this call (the layer before it
        in forward, or after it in the backward recompute); ``all_gather``
        then waits for it instead of issuing its own."""
        if self.world == 1 or self._gloo() or self._prefetched is not None:
            return
        cur = torch.cuda.current_stream(self.device)
        s = _comm_stream(self.device)
        s.wait_stream(cur)  # the shard is final (optimizer of the previous step done)
        with torch.cuda.stream(s):
            full = torch.empty(self.padded, dtype=self.param.dtype, device=self.device)
            dist.all_gather_into_tensor(full, self.param, group=self.group)
            ev = torch.cuda.Event()
            ev.record(s)
        self._prefetched = (full, ev)

    def all_gather(self) -> torch.Tensor:
        if self.world == 1:
            return self.param
        if self._prefetched is not None:
            full, ev = self._prefetched
            self._prefetched = None
            cur = torch.cuda.current_stream(self.device)
            cur.wait_event(ev)
            full.record_stream(cur)
            return full
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


_COMM_STREAMS: dict = {}


def _comm_stream(device: torch.device) -> "torch.cuda.Stream":
    s = _COMM_STREAMS.get(device)
    if s is None:
        s = _COMM_STREAMS[device] = torch.cuda.Stream(device)
    return s


class GradPush:
    """Gradient shards of a set of groups in one symmetric heap (IPC-mapped
    on every rank; a plain device buffer at world 1), plus the barrier flags.

    After construction each group's ``grad`` is a view into this rank's heap
    and ``push_table`` holds every rank's address of that group's shard, so
    kernels can add gradient elements into any owner's shard."""

    def __init__(self, groups: list[FlatGroup], rank: int, world: int, device, group=None):
        from ..parallel.symm import Layout
        self.rank, self.world, self.device, self.group = rank, world, torch.device(device), group
        lay = Layout()
        offs = [lay.add(g.name, (g.shard_n,), torch.float32) for g in groups]
        o_flags = lay.add("flags", (max(world, 1),), torch.int32)
        if world > 1:
            from ..parallel.symm import SymmetricHeap
            self.heap = SymmetricHeap(lay.nbytes, self.device, group)
            view = self.heap.view
            ptrs = self.heap.ptrs
        else:
            self.heap = None
            self._buf = torch.zeros(lay.nbytes // 4, dtype=torch.float32, device=self.device)
            base = self._buf.data_ptr()
            ptrs = [base]

            def view(off, shape, dtype, rank=None):
                n = 1
                for d in shape:
                    n *= int(d)
                return self._buf.view(torch.uint8)[off:off + n * torch.tensor([], dtype=dtype).element_size()] \
                    .view(dtype).view(shape)
        for g, o in zip(groups, offs):
            g.grad = view(o, (g.shard_n,), torch.float32)
            g.grad.zero_()
            g.push_table = torch.tensor([p + o for p in ptrs], dtype=torch.int64, device=self.device)
        self.flags = view(o_flags, (max(world, 1),), torch.int32)
        self.flags.zero_()
        self.peer_flags = torch.tensor([p + o_flags for p in ptrs], dtype=torch.int64, device=self.device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.groups = groups
        torch.cuda.synchronize(self.device)
        if world > 1:
            dist.barrier(group=group)

    def barrier(self):
        """Every rank's pushes issued so far (stream order) are visible in the
        shards once this returns on the stream."""
        from ..ops._ext import ext, scratch
        ext().peer_barrier(self.peer_flags, self.flags, self.epoch, self.rank, self.world,
                           scratch(self.device).status)

    def close(self):
        for g in self.groups:
            g.grad = g.grad.clone()
            g.push_table = None
            g.gathered = (0, 0)
            if g in _PUSH_GROUPS:
                _PUSH_GROUPS.remove(g)
        if self.heap is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.heap.close()
            self.heap = None


def push_target(w: torch.Tensor):
    """(group, flat element offset) when ``w`` is a gathered parameter of a
    push-mode group, else None."""
    ptr = w.data_ptr()
    for fg in _PUSH_GROUPS:
        lo, hi = fg.gathered
        if lo <= ptr < hi:
            return fg, (ptr - lo) // w.element_size()
    return None


_PUSH_GROUPS: list[FlatGroup] = []


class GatherParams(torch.autograd.Function):
    @staticmethod
    def forward(ctx, anchor, fg: FlatGroup):
        ctx.fg = fg
        full = fg.all_gather()
        if fg.push_table is not None:
            ctx.set_materialize_grads(False)  # pushed weight gradients arrive as None
            lo, hi = full.data_ptr(), full.data_ptr() + full.numel() * full.element_size()
            for other in _PUSH_GROUPS:  # a freed gather buffer may have been reused for this one
                if other is not fg and other.gathered[0] < hi and lo < other.gathered[1]:
                    other.gathered = (0, 0)
            fg.gathered = (lo, hi)
            if fg not in _PUSH_GROUPS:
                _PUSH_GROUPS.append(fg)
        return tuple(fg.views(full))

    @staticmethod
    def backward(ctx, *grads):
        fg: FlatGroup = ctx.fg
        if fg.push_table is not None:
            from ..ops._ext import ext
            for g, o in zip(grads, fg.offsets):
                if g is not None:
                    ext().shard_push_add(g.contiguous().view(-1), fg.push_table, o, fg.shard_n, 1.0)
            return None, None
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
