"""Device-resident paged KV cache (block size 16).

Layout per layer: K and V as [num_blocks, num_kv_heads, 16, head_dim] bf16 so
that one page of one kv head is a contiguous [16, head_dim] tile (a pair of
TMA boxes for the attention kernels). All layers live in two tensors
[L, num_blocks, Hkv, 16, D]. A token's cache slot is ``block * 16 + offset``.

Replaces the reference's host-side per-sequence KV snapshots and bucketed
decode buffers (rlx-models-core src/autoregressive.rs:538-1250,
src/gpu_kv.rs:34-590; rlx-serve src/batch.rs:159-300).
"""
from __future__ import annotations

import torch

BLOCK_SIZE = 16


class PagedKVCache:
    """``dtype`` bf16, or torch.float8_e4m3fn: pages then hold saturate(x / s)
    with the per-cache ``scales`` = (s_k, s_v), halving the cache's bytes and
    the decode kernel's reads (prefill reads bf16 copies of its pages)."""

    def __init__(self, num_layers: int, num_blocks: int, num_kv_heads: int, head_dim: int,
                 device: torch.device | str = "cuda", dtype: torch.dtype = torch.bfloat16,
                 scales: tuple = (1.0, 1.0)):
        if dtype not in (torch.bfloat16, torch.float8_e4m3fn):
            raise ValueError(f"KV cache dtype {dtype}: bf16 or float8_e4m3fn")
        self.dtype, self.scales = dtype, (float(scales[0]), float(scales[1]))
        self.num_layers = num_layers
        self.num_blocks = num_blocks
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        shape = (num_layers, num_blocks, num_kv_heads, BLOCK_SIZE, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)

    def layer(self, i: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.k[i], self.v[i]

    @staticmethod
    def bytes_per_block(num_layers: int, num_kv_heads: int, head_dim: int, dtype_bytes: int = 2) -> int:
        return 2 * num_layers * num_kv_heads * BLOCK_SIZE * head_dim * dtype_bytes

    @classmethod
    def blocks_for_memory(cls, mem_bytes: int, num_layers: int, num_kv_heads: int, head_dim: int) -> int:
        return max(1, mem_bytes // cls.bytes_per_block(num_layers, num_kv_heads, head_dim))
