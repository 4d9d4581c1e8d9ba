"""Fused sequence-parallel tensor-parallel communicator (the product TP path).

Residual stream: sharded by token rows; rank q owns rows
[q * rpr, min(M, (q + 1) * rpr)) with rpr = ceil(M / world).

Row-parallel op (o_proj, down_proj)::

    GEMM(x, w_shard) --push rows over NVLink--> owner's recv[slot = my rank]
                     --last CTA--> rs_flags[my rank] = epoch   on every rank
    rs_norm_ag:  wait rs flags; h_shard += sum(recv slots); x_norm = rmsnorm(h) * w
                 push x_norm rows into every rank's gather buffer; ag barrier

so the reduce-scatter rides in the GEMM epilogue (tile by tile, overlapping the
remaining MMAs) and the all-gather rides in the norm kernel. The next
column-parallel GEMM reads the gathered activation from local memory, so every
activation byte crosses NVLink once. No NCCL call sits on this path.

Buffer reuse is safe without double buffering: a rank writes a peer's recv
slot only in op k+1, after that peer's op-k ag barrier, which the peer raises
only after its own op-k reads of recv; a rank's gather buffer is rewritten in
op k+1's norm step only after that rank raised its op-k+1 rs flag, i.e. after
its GEMMs that read the gather buffer (stream order).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .. import ops
from ..ops._ext import ext, scratch
from .symm import Layout, SymmetricHeap
from .tp import NcclTPComm


class FusedTPComm(NcclTPComm):
    name = "fused"

    def __init__(self, rank: int, world: int, device, eps: float = 1e-6, *, max_tokens: int = 8192,
                 hidden: int = 4096, group=None):
        super().__init__(rank, world, device, eps, group)
        self.H = hidden
        self.max_tokens = max_tokens
        self.rpr_max = math.ceil(max_tokens / world)
        lay = Layout()
        self.o_recv = lay.add("recv", (world, self.rpr_max, hidden), torch.bfloat16)
        self.o_gath = lay.add("gath", (max_tokens, hidden), torch.bfloat16)
        self.acc_rows = math.ceil(128 / world)  # decode steps (M <= 128) accumulate in fp32
        self.o_racc = lay.add("racc", (self.acc_rows, hidden), torch.float32)
        # one-shot (decode) path: double-buffered per-rank bf16 slots + flags
        self.os_rows = 128
        self.o_os = lay.add("os_slots", (2, world, self.os_rows, hidden), torch.bfloat16)
        self.o_osf = lay.add("os_flags", (world,), torch.int32)
        self.o_rs = lay.add("rs_flags", (world,), torch.int32)
        self.o_ag = lay.add("ag_flags", (world,), torch.int32)
        self.heap = SymmetricHeap(lay.nbytes, device, group)
        self.recv = self.heap.view(self.o_recv, (world, self.rpr_max, hidden), torch.bfloat16)
        self.gath = self.heap.view(self.o_gath, (max_tokens, hidden), torch.bfloat16)
        self.racc = self.heap.view(self.o_racc, (self.acc_rows, hidden), torch.float32)
        self.peer_racc = self.heap.peer_ptr_table(self.o_racc)
        self.os_slots = self.heap.view(self.o_os, (2, world, self.os_rows, hidden), torch.bfloat16)
        self.os_flags = self.heap.view(self.o_osf, (world,), torch.int32)
        slot_bytes = world * self.os_rows * hidden * 2
        self.peer_os = [self.heap.peer_ptr_table(self.o_os + par * slot_bytes) for par in (0, 1)]
        self.peer_osf = self.heap.peer_ptr_table(self.o_osf)
        self.parity = 0
        self.one_shot = False
        self.rs_flags = self.heap.view(self.o_rs, (world,), torch.int32)
        self.ag_flags = self.heap.view(self.o_ag, (world,), torch.int32)
        self.peer_recv = self.heap.peer_ptr_table(self.o_recv)
        self.peer_gath = self.heap.peer_ptr_table(self.o_gath)
        self.peer_rs = self.heap.peer_ptr_table(self.o_rs)
        self.peer_ag = self.heap.peer_ptr_table(self.o_ag)
        # local counters: [epoch, rs-norm CTA arrivals, GEMM CTA arrivals]
        self.ctr = torch.zeros(3, dtype=torch.int32, device=device)
        self.slot_elems = self.rpr_max * hidden
        self.M = 0
        self.rpr = 0
        dist.barrier(group=group)

    # -- residual-stream contract ---------------------------------------------
    def embed(self, ids, table):
        M = ids.shape[0]
        assert M <= self.max_tokens, f"step of {M} tokens exceeds the TP buffers ({self.max_tokens})"
        self.M = M
        self.parity = 0
        self.one_shot = M <= self.os_rows
        if self.one_shot:
            # decode-sized step: replicated residual stream, one-shot reductions
            return ops.embedding(ids, table)
        self.rpr = math.ceil(M / self.world)
        lo = min(M, self.rank * self.rpr)
        hi = min(M, lo + self.rpr)
        h = torch.empty(self.rpr, table.shape[1], dtype=table.dtype, device=table.device)
        if hi > lo:
            ops.embedding(ids[lo:hi], table, out=h[:hi - lo])
        return h

    def _rs_norm_ag(self, recv, h, norm_w, racc=None):
        s = scratch(h.device)
        ops._count(1)
        ext().rs_norm_ag(recv, racc, h, norm_w, self.peer_gath, self.rs_flags, self.ag_flags, self.peer_ag,
                         self.ctr[0:1], self.ctr[1:2], self.M, self.rpr, self.world, self.rank, self.slot_elems,
                         float(self.eps), s.status)
        return self.gath[:self.M]

    def norm_in(self, h, w):
        if self.one_shot:
            return ops.rmsnorm(h, w, self.eps)
        return self._rs_norm_ag(None, h, w)

    def rowpar_add_norm(self, x, w, h, norm_w, bias=None):
        s = scratch(x.device)
        ops._count(1)
        if self.one_shot:
            # GEMM epilogue broadcasts its bf16 partial rows into slot `rank` of
            # every rank (this op's parity buffer); one kernel per rank waits for
            # all ranks' epoch flags, sums the slots, adds the residual, RMSNorm.
            par = self.parity
            self.parity ^= 1
            ext().linear_push(x, w, bias if self.rank == 0 else None, 0, True, self.M, self.H,
                              self.os_rows * self.H, self.rank, self.world, self.peer_os[par], self.peer_osf,
                              self.ctr[0:1], self.ctr[2:3], s.gemm_ws, s.gemm_sem, s.status)
            out = torch.empty_like(h)
            ops._count(1)
            ext().os_reduce_norm(self.os_slots[par], self.os_rows * self.H, h, norm_w, out, self.os_flags,
                                 self.ctr[0:1], self.ctr[1:2], self.M, self.world, float(self.eps), s.status)
            return out
        if x.shape[0] <= 128 and bias is None:
            # decode: split-K partials red.add'ed straight into the owner's fp32 accumulator
            ext().linear_push(x, w, None, 3, False, self.rpr, self.H, 0, self.rank, self.world, self.peer_racc,
                              self.peer_rs, self.ctr[0:1], self.ctr[2:3], s.gemm_ws, s.gemm_sem, s.status)
            return self._rs_norm_ag(None, h, norm_w, racc=self.racc)
        ext().linear_push(x, w, bias if self.rank == 0 else None, 0, False, self.rpr, self.H, self.slot_elems, self.rank,
                          self.world, self.peer_recv, self.peer_rs, self.ctr[0:1], self.ctr[2:3], s.gemm_ws,
                          s.gemm_sem, s.status)
        return self._rs_norm_ag(self.recv, h, norm_w)

    def close(self):
        self.heap.close()
