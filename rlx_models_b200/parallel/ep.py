"""Expert-parallel combine over NVLink peer memory (the fused EP path).

Expert parallelism with replicated attention: every rank holds the step's
tokens, routes them identically, and runs the grouped MXFP4 GEMMs for its own
``e_local`` experts only. The per-layer MoE output then has to be gathered
from the ranks that own each token's experts. ``EPCombiner`` does that in one
kernel per layer:

    moe_align       writes this rank's inverse permutation into its inv slot
    down GEMM       writes router-weighted expert rows into its rows slot
                    (both slots live in a symmetric IPC heap)
    ep_combine_norm barrier, then per token: read the k expert rows from the
                    owning ranks' HBM over NVLink, sum in slot order,
                    h += moe, out = rmsnorm(h) * w           (one kernel)

No NCCL call sits on this path; the sum has the single-GPU order, so EP = N
reproduces EP = 1 bit for bit. With ``world == 1`` (no process group) the same
kernel runs on plain device buffers and replaces the combine + add + norm
kernels of the single-GPU MoE block.

Slots are double-buffered by op parity. An even number of ops per forward
(one per MoE layer) keeps the parity of every forward identical, so captured
CUDA graphs replay with consistent buffers; ``usable`` is False otherwise and
the model falls back to NCCL.

Reference: the reference's expert parallelism is host TCP expert offload
(crates/rlx-kimi-k3/src/dist_experts.rs:666-757); it has no device-side EP.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..ops._ext import ext, scratch


class EPCombiner:
    def __init__(self, rank: int, world: int, device, *, hidden: int, top_k: int, e_local: int, max_tokens: int,
                 num_layers: int, eps: float, group=None):
        self.rank, self.world, self.device = rank, world, torch.device(device)
        self.H, self.k, self.e_local, self.eps = hidden, top_k, e_local, eps
        self.max_tokens = max_tokens
        self.rows_max = max_tokens * top_k
        self.group = group
        self.usable = num_layers % 2 == 0 or world == 1
        self.parity = 0
        shapes = [("rows", (2, self.rows_max, hidden), torch.bfloat16), ("inv", (2, self.rows_max), torch.int32),
                  ("flags", (max(world, 1),), torch.int32)]
        if world > 1:
            from .symm import Layout, SymmetricHeap
            lay = Layout()
            offs = {n: lay.add(n, s, d) for n, s, d in shapes}
            self.heap = SymmetricHeap(lay.nbytes, self.device, group)
            self.rows = self.heap.view(offs["rows"], shapes[0][1], torch.bfloat16)
            self.inv = self.heap.view(offs["inv"], shapes[1][1], torch.int32)
            self.flags = self.heap.view(offs["flags"], shapes[2][1], torch.int32)
            rb, ib = self.rows_max * hidden * 2, self.rows_max * 4
            self.peer_rows = [self.heap.peer_ptr_table(offs["rows"] + p * rb) for p in (0, 1)]
            self.peer_inv = [self.heap.peer_ptr_table(offs["inv"] + p * ib) for p in (0, 1)]
            self.peer_flags = self.heap.peer_ptr_table(offs["flags"])
        else:
            self.heap = None
            self.rows = torch.zeros(shapes[0][1], dtype=torch.bfloat16, device=self.device)
            self.inv = torch.full(shapes[1][1], -1, dtype=torch.int32, device=self.device)
            self.flags = torch.zeros(1, dtype=torch.int32, device=self.device)
            tab = lambda t: torch.tensor([t.data_ptr()], dtype=torch.int64, device=self.device)  # noqa: E731
            self.peer_rows = [tab(self.rows[p]) for p in (0, 1)]
            self.peer_inv = [tab(self.inv[p]) for p in (0, 1)]
            self.peer_flags = tab(self.flags)
        self.rows.zero_()
        self.inv.fill_(-1)
        self.flags.zero_()
        self.ctr = torch.zeros(2, dtype=torch.int32, device=self.device)  # [epoch, CTA arrivals]
        torch.cuda.synchronize(self.device)
        if world > 1:
            dist.barrier(group=group)

    def fits(self, T: int) -> bool:
        return self.usable and T <= self.max_tokens

    def slots(self, n: int):
        """(rows [n, H], inv [n]) of the next op's parity; the caller's align
        kernel writes inv and its down GEMM writes rows."""
        p = self.parity
        return self.rows[p, :n], self.inv[p, :n]

    def combine_norm(self, experts: torch.Tensor, h: torch.Tensor, norm_w: torch.Tensor) -> torch.Tensor:
        """h += sum over each token's expert rows (any rank); returns rmsnorm(h) * norm_w."""
        p = self.parity
        self.parity ^= 1
        out = torch.empty_like(h)
        s = scratch(h.device)
        ops._count(1)
        ext().ep_combine_norm(self.peer_rows[p], self.peer_inv[p], self.peer_flags, self.flags, experts,
                              self.e_local, h, norm_w, out, self.ctr[0:1], self.ctr[1:2], self.rank, self.world,
                              float(self.eps), s.status)
        return out

    def close(self):
        if self.heap is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.heap.close()
            self.heap = None
