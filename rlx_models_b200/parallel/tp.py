"""Tensor-parallel communicators for the decoder residual stream.

Each communicator implements the residual-stream contract used by
:class:`~rlx_models_b200.models.decoder.DecoderLM`:

* ``embed(ids, table)``         embedding rows this rank keeps,
* ``norm_in(h, w)``             first RMSNorm (and gather, if sharded),
* ``rowpar_add_norm(x, w, h, norm_w, bias)``
                                row-parallel GEMM partial -> reduce over ranks ->
                                residual add into ``h`` -> RMSNorm for the next
                                column-parallel GEMM,
* ``sample(logits_local, ...)`` token choice over vocab-parallel logits.

``NcclTPComm`` is the baseline: replicated residual stream, our GEMM for the
partial, ``torch.distributed.all_reduce`` (NCCL) for the sum, our fused
add+RMSNorm kernel after it. ``FusedTPComm`` (parallel/fused_tp.py) is the
product path: the GEMM epilogue pushes partial tiles over NVLink into the
owner rank's receive buffer (reduce-scatter fused into the GEMM), and one
kernel does reduce + residual + RMSNorm + all-gather over peer memory.

The reference has no tensor-parallel model path (its TP prototype lives in an
external crate, docs/distributed-inference-design.md:596-652).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops


class NcclTPComm:
    """Baseline TP communicator: NCCL all-reduce between our kernels."""

    name = "nccl"

    def __init__(self, rank: int, world: int, device: torch.device, eps: float = 1e-6, group=None):
        self.rank, self.world, self.device, self.eps = rank, world, device, eps
        self.group = group
        # second communicator on its own process group for overlapped prefill
        # micro-batches (models.decoder.DecoderLM._forward_overlapped); None = off
        self.microbatch_comm = None

    def embed(self, ids, table):
        return ops.embedding(ids, table)

    def norm_in(self, h, w):
        return ops.rmsnorm(h, w, self.eps)

    def rowpar_add_norm(self, x, w, h, norm_w, bias=None):
        if x.shape[0] <= ops.ACC_MAX_M and bias is None:
            # decode: fp32 partial from the accumulate-only GEMM, NCCL sum, then
            # one kernel does h += sum, rmsnorm and re-zeroes the accumulator
            part = ops.linear_acc(x, w)
            dist.all_reduce(part, group=self.group)
            return ops.add_rmsnorm_acc(part, h, norm_w, self.eps)
        part = ops.linear(x, w, bias=bias if self.rank == 0 else None)
        dist.all_reduce(part, group=self.group)
        # h = h + part ; return rmsnorm(h) * norm_w   (one fused kernel)
        return ops.rmsnorm(part, norm_w, self.eps, residual=h, residual_out=h)

    # -- vocab-parallel token selection ---------------------------------------
    def gather_logits(self, logits_local: torch.Tensor) -> torch.Tensor:
        """[R, V/world] -> [R, V] on every rank."""
        R, Vl = logits_local.shape
        buf = torch.empty(self.world, R, Vl, dtype=logits_local.dtype, device=logits_local.device)
        dist.all_gather_into_tensor(buf, logits_local.contiguous(), group=self.group)
        return buf.permute(1, 0, 2).reshape(R, self.world * Vl)

    def greedy(self, logits_local: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Global argmax over vocab shards: local argmax, then an all-gather of
        (value, global index) pairs; ties resolve to the lowest index."""
        R, Vl = logits_local.shape
        idx = ops.argmax(logits_local)
        val = logits_local.gather(1, idx.long().unsqueeze(1)).squeeze(1)
        pair = torch.stack([val, (idx.float() + float(self.rank * Vl))], dim=1)  # exact for V < 2^24
        allp = torch.empty(self.world, R, 2, dtype=pair.dtype, device=pair.device)
        dist.all_gather_into_tensor(allp, pair, group=self.group)
        best = allp[:, :, 0].argmax(0)  # first rank with the max value = lowest index
        out.copy_(allp[best, torch.arange(R, device=pair.device), 1].to(torch.int32))
        return out


def make_tp_comm(kind: str, rank: int, world: int, device, eps: float = 1e-6, prefill_overlap: bool | None = None,
                 **kw):
    """``prefill_overlap`` (default: on unless B200_TP_PREFILL_OVERLAP=0) gives the
    NCCL and pull communicators a second NCCL process group, so large prefill
    steps run as two micro-batches whose all-reduces overlap each other's compute."""
    if world == 1:
        return None
    if kind == "nccl":
        comm = NcclTPComm(rank, world, device, eps)
    elif kind == "fused":
        from .fused_tp import FusedTPComm
        return FusedTPComm(rank, world, device, eps, **kw)
    elif kind == "pull":
        from .pull_tp import PullTPComm
        comm = PullTPComm(rank, world, device, eps, **kw)
    else:
        raise ValueError(kind)
    if prefill_overlap is None:
        from .. import settings
        prefill_overlap = settings.get("B200_TP_PREFILL_OVERLAP")
    if prefill_overlap:
        g2 = dist.new_group(list(range(world)))
        comm.microbatch_comm = NcclTPComm(rank, world, device, eps, group=g2)
    return comm
