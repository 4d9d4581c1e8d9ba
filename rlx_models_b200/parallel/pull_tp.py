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

From 4 ranks and 16 rows up (``two_shot``), the reduction is two-shot
(``ar2_norm``): each rank reduces and normalises only the rows it owns and the
others copy the finished rows, so a rank reads M*H*4/world bytes of partials
instead of M*H*4*(world-1), at the price of a second flag barrier.
Token choice over the vocab-parallel logits is one peer-memory kernel
(``PeerArgmax``) instead of an NCCL all-gather.

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


class PeerArgmax:
    """Vocab-parallel greedy choice in one kernel over NVLink peer memory
    (``csrc/comm/tp_sample.cu``): local shard argmax packed into a key that
    carries its op's tag, pushed into every rank's key buffer, polled by tag
    (no flags, no fences); every rank gets the global argmax (lowest index on
    ties). Replaces the local argmax + NCCL all-gather + selection of the
    baseline communicator."""

    def __init__(self, rank: int, world: int, device, max_rows: int = 256, group=None):
        self.rank, self.world, self.max_rows = rank, world, max_rows
        lay = Layout()
        o_keys = lay.add("keys", (2, max_rows, world), torch.int64)
        self.heap = SymmetricHeap(lay.nbytes, device, group)
        self.keys = self.heap.view(o_keys, (2, max_rows, world), torch.int64)
        self.keys.zero_()
        self.peer_keys = self.heap.peer_ptr_table(o_keys)
        self.ctr = torch.zeros(2, dtype=torch.int32, device=device)  # [epoch, departures]
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def __call__(self, logits_local: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        R, Vl = logits_local.shape
        if R > self.max_rows:
            raise ValueError(f"PeerArgmax: {R} rows > {self.max_rows}")
        ops._count(1)
        ext().tp_argmax(logits_local, self.rank * Vl, self.keys, self.peer_keys, self.ctr[0:1], self.ctr[1:2], out,
                        self.max_rows, self.rank, self.world, scratch(logits_local.device).status)
        return out

    def close(self):
        self.heap.close()


class PullTPComm(NcclTPComm):
    name = "pull"
    ROWS = 128

    def __init__(self, rank: int, world: int, device, eps: float = 1e-6, *, hidden: int = 4096, group=None,
                 two_shot: str | None = None, **kw):
        super().__init__(rank, world, device, eps, group)
        self.H = hidden
        # "auto": two-shot from 8 ranks and 16 rows (at 4 ranks the one-shot pull measured
        # 28.3 vs 34.0 us per GEMM + reduction at 64 rows; at 8, 48.7 vs 41.5); "on" / "off" force it
        from .. import settings
        self.two_shot = two_shot or settings.get("B200_TP_TWO_SHOT")
        self.rpr_max = (self.ROWS + world - 1) // world
        lay = Layout()
        self.o_acc = lay.add("acc", (2, self.ROWS, hidden), torch.float32)
        self.o_flags = lay.add("flags", (world,), torch.int32)
        self.o_res = lay.add("res", (2, self.rpr_max, hidden), torch.bfloat16)
        self.o_flags2 = lay.add("flags2", (2, world), torch.int32)
        self.heap = SymmetricHeap(lay.nbytes, device, group)
        self.acc = self.heap.view(self.o_acc, (2, self.ROWS, hidden), torch.float32)
        self.acc.zero_()
        self.flags = self.heap.view(self.o_flags, (world,), torch.int32)
        self.flags.zero_()
        slot = self.ROWS * hidden * 4
        self.peer_acc = [self.heap.peer_ptr_table(self.o_acc + p * slot) for p in (0, 1)]
        self.peer_flags = self.heap.peer_ptr_table(self.o_flags)
        self.res = self.heap.view(self.o_res, (2, self.rpr_max, hidden), torch.bfloat16)
        self.flags2 = self.heap.view(self.o_flags2, (2, world), torch.int32)
        self.flags2.zero_()
        self.peer_res = self.heap.peer_ptr_table(self.o_res)
        self.peer_flags2 = self.heap.peer_ptr_table(self.o_flags2)
        self.ctr2 = torch.zeros(3, dtype=torch.int32, device=device)  # two-shot [epoch, arrivals, departures]
        self.ctr = torch.zeros(2, dtype=torch.int32, device=device)  # [epoch, CTA arrivals]
        self.parity = 0
        self.argmax = PeerArgmax(rank, world, device, max_rows=256, group=group)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def _use_two_shot(self, M: int) -> bool:
        if self.two_shot == "on":
            return True
        if self.two_shot == "off":
            return False
        return self.world >= 8 and M >= 16

    def greedy(self, logits_local: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        if logits_local.shape[0] > self.argmax.max_rows:
            return super().greedy(logits_local, out)
        return self.argmax(logits_local, out)

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
        if self._use_two_shot(M):
            rpr = (M + self.world - 1) // self.world
            ext().ar2_norm(self.peer_acc[p], self.peer_res, self.res, self.peer_flags2, self.flags2, self.acc[p ^ 1],
                           self.ROWS, h, norm_w, out, self.ctr2[0:1], self.ctr2[1:3], self.rank, self.world, rpr,
                           self.rpr_max, float(self.eps), s.status)
            return out
        ext().ar_pull_norm(self.peer_acc[p], self.peer_flags, self.flags, self.acc[p ^ 1], self.ROWS, h, norm_w,
                           out, self.ctr[0:1], self.ctr[1:2], self.rank, self.world, float(self.eps), s.status)
        return out

    def close(self):
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self.heap.close()
        self.argmax.close()
