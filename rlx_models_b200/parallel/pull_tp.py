"""Tensor-parallel communicator with a pull all-reduce for decode steps.

Decode-sized steps (M <= 128, no bias) keep the replicated residual stream of
the NCCL communicator, but replace ``linear_acc -> NCCL all_reduce ->
add_rmsnorm_acc`` with

    linear_acc into this rank's fp32 slot of a symmetric (IPC) heap     (local)
    ar_pull_norm: announce, wait for all ranks, read every rank's partial
                  over NVLink, add the residual, RMSNorm                  (1 kernel)

Slots are double-buffered by op parity: the pull kernel of op n zeroes this
rank's op n-1 slot (all ranks have passed op n's barrier, so they are done
reading it) for the GEMM of op n+1. There are 2 row-parallel ops per layer,
so a decode step always ends on the parity it started with, and a captured
CUDA graph replays with consistent buffers. Larger steps (prefill) use NCCL.

Reference: the reference has no tensor-parallel serving path; its collective
design notes (docs/distributed-inference-design.md:596-652) describe the
Megatron split this implements.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..ops._ext import ext, scratch
from .symm import Layout, SymmetricHeap
from .tp import NcclTPComm


class PullTPComm(NcclTPComm):
    name = "pull"
    ROWS = 128

    def __init__(self, rank: int, world: int, device, eps: float = 1e-6, *, hidden: int = 4096, group=None, **kw):
        super().__init__(rank, world, device, eps, group)
        self.H = hidden
        lay = Layout()
        self.o_acc = lay.add("acc", (2, self.ROWS, hidden), torch.float32)
        self.o_flags = lay.add("flags", (world,), torch.int32)
        self.heap = SymmetricHeap(lay.nbytes, device, group)
        self.acc = self.heap.view(self.o_acc, (2, self.ROWS, hidden), torch.float32)
        self.acc.zero_()
        self.flags = self.heap.view(self.o_flags, (world,), torch.int32)
        self.flags.zero_()
        slot = self.ROWS * hidden * 4
        self.peer_acc = [self.heap.peer_ptr_table(self.o_acc + p * slot) for p in (0, 1)]
        self.peer_flags = self.heap.peer_ptr_table(self.o_flags)
        self.ctr = torch.zeros(2, dtype=torch.int32, device=device)  # [epoch, CTA arrivals]
        self.parity = 0
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def rowpar_add_norm(self, x, w, h, norm_w, bias=None):
        M = x.shape[0]
        if M > self.ROWS or bias is not None:
            return super().rowpar_add_norm(x, w, h, norm_w, bias)
        p = self.parity
        self.parity ^= 1
        ops.linear_acc(x, w, acc=self.acc[p, :M])
        out = torch.empty_like(h)
        s = scratch(x.device)
        ops._count(1)
        ext().ar_pull_norm(self.peer_acc[p], self.peer_flags, self.flags, self.acc[p ^ 1], self.ROWS, h, norm_w,
                           out, self.ctr[0:1], self.ctr[1:2], self.rank, self.world, float(self.eps), s.status)
        return out

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.heap.close()
