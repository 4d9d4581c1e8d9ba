"""Pipeline-parallel training with a 1F1B schedule.

Stage ``r`` of ``S`` (one process each) holds a contiguous layer range
(`parallel/pp_plan.py` or an even split); stage 0 also holds the token
embedding, the last stage the final norm and the LM head (its own copy of the
embedding when the model ties them). A step splits this stage's batch into
``M`` micro-batches and runs the one-forward-one-backward schedule:

    warm-up: S - r - 1 forwards; steady state: forward m + w, backward m;
    cool-down: the remaining backwards,

so at most S - r micro-batches of activations are alive on stage r (GPipe
keeps all M). Hidden states go forward and their gradients backward as
point-to-point messages (NCCL on GPUs, gloo on CPU); sends are non-blocking,
receives block, which keeps any interleaving of the ranks deadlock-free.

After the last backward: the tied embedding's gradient is summed between the
first and last stage, the global gradient norm is one all-reduce of per-stage
sums of squares (the tied copy counted once), and every stage applies the same
clipped AdamW as the data-parallel trainer to its own parameters. The result
equals the single-process trainer on the same global batch.

Reference: the reference's pipeline training is GPipe over an RPC transport
(crates/rlx-kimi-k3/src/dist.rs:788-1135, TRAIN_FWD / TRAIN_BWD / GRAD_SQ /
APPLY messages); its pipeline serving splits layers with
`pipeline_layer_range` (docs/distributed-inference-design.md:289-325).
"""
from __future__ import annotations

import math
import time

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .. import ops
from ..ops import rope_inv_freq
from . import functional as TF
from .fsdp import FlatGroup, gather_params
from .model import TrainableDecoder, _layer_tensors
from .trainer import StepMetrics, TrainConfig


def even_ranges(num_layers: int, stages: int) -> list[tuple[int, int]]:
    base, rem = divmod(num_layers, stages)
    out, lo = [], 0
    for s in range(stages):
        hi = lo + base + (1 if s < rem else 0)
        out.append((lo, hi))
        lo = hi
    return out


class StageDecoder(TrainableDecoder):
    """The layers [lo, hi) of a trainable decoder plus the end-stage extras."""

    def __init__(self, cfg, weights, stage: int, stages: int, lo: int, hi: int, device="cpu",
                 param_dtype: torch.dtype = torch.bfloat16, max_seq: int = 8192):
        self.cfg = cfg
        self.device = torch.device(device)
        self.ckpt = False
        self.lora = None
        self.stage, self.stages, self.lo, self.hi = stage, stages, lo, hi
        self.first, self.last = stage == 0, stage == stages - 1

        def get(name):
            t = weights.take(name) if hasattr(weights, "take") else weights[name]
            return t.to(self.device)

        grp = lambda name, named: FlatGroup(name, named, 0, 1, self.device, None, param_dtype)  # noqa: E731
        self.embed_g = grp("embed", [("model.embed_tokens.weight", get("model.embed_tokens.weight"))]) \
            if self.first else None
        self.head_g = None
        if self.last:
            head = get("model.embed_tokens.weight" if cfg.tie_word_embeddings else "lm_head.weight")
            self.head_g = grp("head", [("lm_head.weight", head)])
            self.norm_g = grp("norm", [("model.norm.weight", get("model.norm.weight"))])
        self.layers = [grp(f"layer{i}", _layer_tensors(cfg, i, get)) for i in range(lo, hi)]
        inv, mult = rope_inv_freq(cfg.rotary_dim, cfg.rope_theta, cfg.rope_scaling, cfg.max_position_embeddings)
        freqs = torch.outer(torch.arange(max_seq, dtype=torch.float32), inv)
        emb = torch.cat([freqs, freqs], -1)
        self.cos = (emb.cos() * mult).to(self.device, torch.bfloat16)  # the same tables as TrainableDecoder
        self.sin = (emb.sin() * mult).to(self.device, torch.bfloat16)

    @property
    def groups(self) -> list[FlatGroup]:
        g = ([self.embed_g] if self.first else []) + self.layers
        if self.last:
            g += [self.norm_g, self.head_g]
        return g

    def forward_stage(self, x: torch.Tensor, targets=None, denom=None):
        """Stage 0: x = token ids; otherwise x = the previous stage's hidden
        states. Returns hidden states, or (last stage) the scaled loss."""
        h = F.embedding(x, gather_params(self.embed_g)[0]) if self.first else x
        for i in range(len(self.layers)):
            h = self._layer(h, i)
        if not self.last:
            return h
        norm = gather_params(self.norm_g)[0]
        head = gather_params(self.head_g)[0]
        xn = TF.rmsnorm(h, norm, self.cfg.rms_norm_eps)
        return TF.lm_head_ce(xn.reshape(-1, self.cfg.hidden_size), head, targets.reshape(-1), 2048, denom)


class PipelineTrainer:
    def __init__(self, model_cfg, train_cfg: TrainConfig, weights, stage: int, stages: int, device="cpu",
                 ranges: list[tuple[int, int]] | None = None, group=None, ranks: list[int] | None = None):
        self.cfg = train_cfg
        self.stage, self.stages, self.group = stage, stages, group
        self.ranks = ranks or list(range(stages))
        self.device = torch.device(device)
        ranges = ranges or even_ranges(model_cfg.num_hidden_layers, stages)
        lo, hi = ranges[stage]
        self.model = StageDecoder(model_cfg, weights, stage, stages, lo, hi, self.device,
                                  getattr(torch, train_cfg.param_dtype))
        self.tied = bool(model_cfg.tie_word_embeddings) and stages > 1
        # every rank creates the (first, last) group, as new_group requires
        self.tie_group = dist.new_group([self.ranks[0], self.ranks[-1]]) if self.tied else None
        self.step_num = 0
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._coef = torch.ones(1, dtype=torch.float32, device=self.device)
        self.act_dtype = getattr(torch, train_cfg.param_dtype)

    def _peer(self, s: int) -> int:
        return self.ranks[s]

    def step(self, batch: torch.Tensor) -> StepMetrics:
        """``batch``: the global batch [B, S + 1] (every stage sees it: stage 0
        reads the inputs, the last stage the targets)."""
        t0 = time.perf_counter()
        c, m = self.cfg, self.model
        batch = batch.to(self.device)
        ids, tgt = batch[:, :-1].contiguous(), batch[:, 1:].contiguous()
        B, S = ids.shape
        mb = max(1, c.micro_batch)
        M = math.ceil(B / mb)
        denom = max(1.0, float((tgt >= 0).sum()))
        H = m.cfg.hidden_size
        r, Sg = self.stage, self.stages
        inputs, outputs, sends = {}, {}, []
        total = torch.zeros((), dtype=torch.float32, device=self.device)

        def rows(k):
            return slice(k * mb, min(B, (k + 1) * mb))

        def fwd(k):
            nonlocal total
            sl = rows(k)
            if m.first:
                x = ids[sl]
            else:
                x = torch.empty(sl.stop - sl.start, S, H, dtype=self.act_dtype, device=self.device)
                dist.recv(x, src=self._peer(r - 1), group=self.group)
                x.requires_grad_(True)
            inputs[k] = x
            y = m.forward_stage(x, tgt[sl] if m.last else None, denom)
            if m.last:
                total += y.detach()
            else:
                sends.append(dist.isend(y.detach().contiguous(), dst=self._peer(r + 1), group=self.group))
            outputs[k] = y

        def bwd(k):
            y = outputs.pop(k)
            if m.last:
                y.backward()
            else:
                g = torch.empty_like(y)
                dist.recv(g, src=self._peer(r + 1), group=self.group)
                y.backward(g)
            x = inputs.pop(k)
            if not m.first:
                sends.append(dist.isend(x.grad.contiguous(), dst=self._peer(r - 1), group=self.group))

        warm = min(Sg - r - 1, M)
        for k in range(warm):
            fwd(k)
        for k in range(M - warm):
            fwd(warm + k)
            bwd(k)
        for k in range(M - warm, M):
            bwd(k)
        for h in sends:
            h.wait()
        # loss lives on the last stage; share it
        dist.broadcast(total, src=self._peer(Sg - 1), group=self.group)
        if self.tied and (m.first or m.last):  # both hold copies of the tied embedding: sum their gradients
            gr = m.embed_g.grad if m.first else m.head_g.grad
            dist.all_reduce(gr, group=self.tie_group)
        gnorm = self._clip_coef()
        lr = c.lr_at(self.step_num)
        self.step_num += 1
        for g in m.groups:
            self._adamw(g, lr)
            g.grad.zero_()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        ms = (time.perf_counter() - t0) * 1e3
        return StepMetrics(self.step_num, float(total.item()), float(gnorm.item()), lr, int(denom), ms)

    def _clip_coef(self) -> torch.Tensor:
        m = self.model
        self._sumsq.zero_()
        for g in m.groups:
            if self.tied and m.last and g is m.head_g:
                continue  # the tied embedding is counted once, on the first stage
            if g.grad.is_cuda:
                ops.ext().sumsq(g.grad, self._sumsq)
            else:
                self._sumsq += g.grad.float().pow(2).sum()
        dist.all_reduce(self._sumsq, group=self.group)
        norm = self._sumsq.sqrt()
        if self.cfg.grad_clip and self.cfg.grad_clip > 0:
            torch.clamp(self.cfg.grad_clip / (norm + 1e-6), max=1.0, out=self._coef)
        else:
            self._coef.fill_(1.0)
        return norm

    def _adamw(self, g: FlatGroup, lr: float):
        from .trainer import Trainer
        Trainer._adamw(self, g, lr)  # same update as the data-parallel trainer

    def named_parameters(self) -> dict[str, torch.Tensor]:
        """This stage's fp32 masters under the training names (fused q|k|v and
        gate|up rows, global layer indices; the last stage's head copy is
        ``lm_head.weight``)."""
        out = {}
        for g in self.model.groups:
            out.update(g.named_full())
        return out
