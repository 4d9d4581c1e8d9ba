"""Symmetric device memory across the ranks of a process group.

Every rank allocates one raw device buffer of the same size (outside torch's
caching allocator), exports a CUDA IPC handle, all-gathers the handles over
the process group and maps every peer's buffer into its own address space
(peer access over NVLink / NVSwitch). Kernels then address any rank's copy
with a plain pointer: P2P loads and stores, no multicast.

This is the B200 replacement for the reference's one-sided
`SymmetricTransport` (put / get / barrier over a symmetric heap, external
rlx-driver crate; docs/distributed-inference-design.md:75-95).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext


class SymmetricHeap:
    def __init__(self, nbytes: int, device: torch.device, group=None):
        self.device = torch.device(device)
        self.dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.nbytes = int((nbytes + 4095) // 4096 * 4096)
        C = ext()
        self.local = C.symm_malloc(self.nbytes, self.dev)
        handle = C.ipc_handle(self.local, self.dev)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = []
        for r, h in enumerate(handles):
            self.ptrs.append(self.local if r == self.rank else C.ipc_open(h, self.dev))
        self._closed = False

    def view(self, offset: int, shape, dtype: torch.dtype, rank: int | None = None) -> torch.Tensor:
        """Tensor view of [offset, offset + numel) bytes in ``rank``'s buffer (default: own)."""
        r = self.rank if rank is None else rank
        numel = 1
        for s in shape:
            numel *= int(s)
        assert offset + numel * torch.tensor([], dtype=dtype).element_size() <= self.nbytes
        return ext().tensor_from_ptr(self.ptrs[r] + offset, list(shape), dtype, self.dev)

    def peer_ptr_table(self, offset: int) -> torch.Tensor:
        """Device int64 [world] array of each rank's address of ``offset``."""
        return torch.tensor([p + offset for p in self.ptrs], dtype=torch.int64, device=self.device)

    def close(self):
        if self._closed:
            return
        C = ext()
        torch.cuda.synchronize(self.device)
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                C.ipc_close(p, self.dev)
        C.symm_free(self.local, self.dev)
        self._closed = True


class Layout:
    """Byte-offset allocator inside one symmetric buffer (256-byte aligned)."""

    def __init__(self):
        self.off = 0
        self.items: dict[str, tuple[int, tuple, torch.dtype]] = {}

    def add(self, name: str, shape, dtype: torch.dtype) -> int:
        numel = 1
        for s in shape:
            numel *= int(s)
        nb = numel * torch.tensor([], dtype=dtype).element_size()
        self.off = (self.off + 255) // 256 * 256
        self.items[name] = (self.off, tuple(shape), dtype)
        self.off += nb
        return self.items[name][0]

    @property
    def nbytes(self) -> int:
        return (self.off + 255) // 256 * 256
