"""Pipeline parallelism for serving: contiguous layer ranges per rank, the
residual stream relayed stage to stage with NCCL send/recv.

Stage r holds layers [l0, l1) (as a DecoderLM over a remapped weight view, so
its KV cache covers only its layers); stage 0 embeds, the last stage applies
the final norm and lm_head and samples; the sampled tokens are broadcast from
the last stage so every rank's scheduler (identical on all ranks) advances in
lockstep. Each step moves T x hidden bf16 between neighbours.

Reference: rlx-qwen3 src/pipeline.rs, src/pipeline_block.rs:436 (stage
split and hidden-state relay; the reference relays over TCP, here NCCL p2p
over NVLink).
"""
from __future__ import annotations

import dataclasses
import re

import torch
import torch.distributed as dist

from ..models.decoder import DecoderLM, LocalComm

_LAYER = re.compile(r"^model\.layers\.(\d+)\.")


class _LayerView:
    """Weight source whose layer j is the underlying layer j + offset."""

    def __init__(self, w, offset: int):
        self.w, self.off = w, offset

    def _map(self, name):
        m = _LAYER.match(name)
        if not m:
            return name
        return f"model.layers.{int(m.group(1)) + self.off}." + name[m.end():]

    def __contains__(self, name):
        return self._map(name) in self.w

    def __getitem__(self, name):
        return self.w[self._map(name)]

    def take(self, name, **kw):
        return self.w.take(self._map(name), **kw) if hasattr(self.w, "take") else self.w[self._map(name)]

    def take_shard(self, name, *a, **kw):
        return self.w.take_shard(self._map(name), *a, **kw)

    def keys(self):
        return list(self.w.keys())


def stage_layers(num_layers: int, pp_rank: int, pp_size: int) -> tuple[int, int]:
    base, rem = divmod(num_layers, pp_size)
    lo = pp_rank * base + min(pp_rank, rem)
    return lo, lo + base + (1 if pp_rank < rem else 0)


class PipelineDecoderLM(DecoderLM):
    def __init__(self, cfg, weights, device="cuda", pp_rank: int = 0, pp_size: int = 1, group=None,
                 ranks: list[int] | None = None):
        lo, hi = stage_layers(cfg.num_hidden_layers, pp_rank, pp_size)
        self.full_cfg = cfg
        self.pp_rank, self.pp_size, self.pp_group = pp_rank, pp_size, group
        self.pp_ranks = ranks or list(range(pp_size))  # global rank of each stage
        self.layer_range = (lo, hi)
        super().__init__(dataclasses.replace(cfg, num_hidden_layers=hi - lo), _LayerView(weights, lo), device=device)

    @property
    def is_last(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    def forward(self, fb, kv):
        comm = LocalComm(self.cfg.rms_norm_eps)
        T = fb.num_tokens
        if self.pp_rank == 0:
            h = comm.embed(fb.input_ids, self.embed)
            if self.cfg.embedding_multiplier != 1.0:
                h.mul_(self.cfg.embedding_multiplier)
        else:
            h = torch.empty(T, self.cfg.hidden_size, dtype=torch.bfloat16, device=self.device)
            dist.recv(h, src=self.pp_ranks[self.pp_rank - 1], group=self.pp_group)
        x = comm.norm_in(h, self.layers[0].ln1)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            x = self._layer(i, L, x, h, fb, kv, comm, self.layers[i + 1].ln1 if i + 1 < n else self.norm)
        if not self.is_last:
            dist.send(h, dst=self.pp_ranks[self.pp_rank + 1], group=self.pp_group)
            return None
        if fb.logit_rows is not None:
            x = x.index_select(0, fb.logit_rows)
        return self.logits(x)

    def share_tokens(self, toks: torch.Tensor) -> torch.Tensor:
        """Broadcast the last stage's sampled tokens to every stage (in place)."""
        dist.broadcast(toks, src=self.pp_ranks[-1], group=self.pp_group)
        return toks
