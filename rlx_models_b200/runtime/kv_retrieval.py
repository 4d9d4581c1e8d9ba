"""Retrieval over the paged KV cache for long-context decode.

Each decode step attends to a fixed number of KV blocks per sequence instead
of the whole context: the first ``sink_blocks`` blocks, the last
``window_blocks`` blocks (which include the partial current block) and the
``topk_blocks`` older blocks whose key summaries score highest against the
step's query. A block's summary is the mean of its 16 (rotated) keys per KV
head, refreshed for every block written in a step; the score of a block is
sum over KV heads and their query heads of q . summary.

Keys in the cache already carry RoPE at their original positions, so a
selected block enters attention unchanged: the selection is a per-sequence
block table (kept in block order) plus a context length whose last block is
the partial one, fed to the same paged decode kernel. The cost of a decode
step is bounded by (sink + window + topk) blocks whatever the context length.

B200 design: everything stays in HBM. The summaries of a 1M-token context
(62.5k blocks x KV heads x head_dim bf16 per layer) are read by one batched
GEMM per layer, a few microseconds at HBM bandwidth, so the exact top-k over
all blocks replaces the reference's approximate HNSW index (which exists to
search host / disk tiers on a laptop-class machine). Selection uses static
shapes (topk over the table width), so it is captured in the decode CUDA
graphs.

Reference: crates/rlx-qwen3 src/generator.rs:421-660,952-1140 (disk-tiered
HNSW KV context store: evict old rows, retrieve top-k relevant blocks,
splice them RoPE-correctly into past K / V); docs/qwen3-decode-optimization.md:93-118.
"""
from __future__ import annotations

import torch

from .kv_cache import BLOCK_SIZE


class KVRetrieval:
    def __init__(self, num_layers: int, num_blocks: int, num_kv_heads: int, head_dim: int, device,
                 topk_blocks: int = 64, window_blocks: int = 16, sink_blocks: int = 1):
        self.topk, self.window, self.sink = int(topk_blocks), int(window_blocks), int(sink_blocks)
        self.budget = self.topk + self.window + self.sink
        self.summ = torch.zeros(num_layers, num_blocks, num_kv_heads, head_dim, dtype=torch.bfloat16, device=device)

    def update(self, layer: int, k_cache: torch.Tensor, slots: torch.Tensor):
        """Refresh the summaries of the blocks written this step (k_cache
        [blocks, Hkv, 16, D]; slots [T] token cache slots)."""
        if k_cache.is_cuda:
            from .. import ops
            from ..ops._ext import ext
            ext().kv_summary(k_cache, slots.contiguous(), self.summ[layer])
            ops._count(1)
            return
        blk = torch.div(slots, BLOCK_SIZE, rounding_mode="floor")
        self.summ[layer].index_copy_(0, blk, k_cache.index_select(0, blk).float().mean(2).to(torch.bfloat16))

    def select(self, layer: int, q: torch.Tensor, tables: torch.Tensor, ctx: torch.Tensor):
        """q [B, Hq, D] decode queries, tables [B, W], ctx [B] ->
        (selected tables [B, budget] int32, their context lengths [B] int32).
        With a budget of at least the sequence's block count every block is kept."""
        B, W = tables.shape
        Hkv, D = self.summ.shape[2], self.summ.shape[3]
        if self.budget >= W:
            return tables, ctx
        if q.is_cuda:  # block scores (many CTAs), then radix top-k + ordered table + context length
            from .. import ops
            from ..ops._ext import ext
            sel = torch.empty(B, self.budget, dtype=torch.int32, device=q.device)
            sctx = torch.empty(B, dtype=torch.int32, device=q.device)
            scores = torch.empty(B, W, dtype=torch.float32, device=q.device)
            ext().kv_select(q.contiguous(), self.summ[layer], tables.contiguous(), ctx, scores, sel, sctx,
                            self.topk, self.window, self.sink)
            ops._count(2)
            return sel, sctx
        return self.select_reference(layer, q, tables, ctx)

    def select_reference(self, layer: int, q: torch.Tensor, tables: torch.Tensor, ctx: torch.Tensor):
        """torch restatement of the selection kernel (any device)."""
        B, W = tables.shape
        Hkv, D = self.summ.shape[2], self.summ.shape[3]
        s = self.summ[layer].index_select(0, tables.reshape(-1).long()).view(B, W, Hkv, D)
        qg = q.view(B, Hkv, -1, D).sum(2)  # sum over the query heads of each KV head
        score = torch.einsum("bhd,bwhd->bw", qg.float(), s.float())
        ctx = ctx.long()
        nblk = torch.div(ctx + BLOCK_SIZE - 1, BLOCK_SIZE, rounding_mode="floor")
        w = torch.arange(W, device=tables.device)[None, :]
        keep = (w < self.sink) | (w >= nblk[:, None] - self.window)
        score = torch.where(keep, torch.full_like(score, float("inf")), score)
        score = score.masked_fill(w >= nblk[:, None], float("-inf"))
        idx = score.topk(self.budget, dim=1).indices.sort(dim=1).values
        sel = tables.gather(1, idx)
        n_sel = torch.minimum(nblk, torch.full_like(nblk, self.budget))
        last = ctx - (nblk - 1) * BLOCK_SIZE  # tokens in the partial (last) block
        return sel.to(torch.int32), ((n_sel - 1) * BLOCK_SIZE + last).to(torch.int32)
