"""FSDP trainer: gradient accumulation, global-norm clipping, fused AdamW,
LR schedules and world-size-agnostic sharded checkpoints.

Mirrors the knobs of the reference trainer (rlx-tune src/trainer.rs:
`AdamConfig` :273-320, `LrSchedule` + `DpConfig` :439-690 with warmup,
cosine/linear decay, grad_accum, clip; `StepMetrics` :695; checkpoint /
restore :1247-1400, which gathers ZeRO shards so a checkpoint can be resumed
at any world size). Here the optimizer state never leaves the GPUs: each rank
updates its own shard with one fused kernel per parameter group.
"""
from __future__ import annotations

import json
import math
import os
import time
from dataclasses import asdict, dataclass, field

import torch
import torch.distributed as dist

from .. import ops
from ..weights.safetensors_io import Checkpoint, save_file
from .fsdp import FlatGroup
from .model import TrainableDecoder


@dataclass
class TrainConfig:
    lr: float = 1e-4
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.1
    grad_clip: float = 1.0
    schedule: str = "constant"  # constant | cosine | linear
    warmup_steps: int = 0
    total_steps: int = 20
    min_lr_ratio: float = 0.1
    micro_batch: int = 1        # sequences per micro-step per rank
    activation_checkpointing: bool = True
    param_dtype: str = "bfloat16"  # float32 only for exactness tests

    def lr_at(self, step: int) -> float:
        if self.warmup_steps and step < self.warmup_steps:
            return self.lr * (step + 1) / self.warmup_steps
        if self.schedule == "constant":
            return self.lr
        frac = min(1.0, (step - self.warmup_steps) / max(1, self.total_steps - self.warmup_steps))
        lo = self.lr * self.min_lr_ratio
        if self.schedule == "cosine":
            return lo + 0.5 * (self.lr - lo) * (1 + math.cos(math.pi * frac))
        return self.lr - (self.lr - lo) * frac


@dataclass
class StepMetrics:
    step: int
    loss: float
    grad_norm: float
    lr: float
    tokens: int
    step_ms: float

    def __str__(self):
        return (f"step {self.step} loss {self.loss:.4f} |g| {self.grad_norm:.3f} lr {self.lr:.2e} "
                f"{self.tokens / max(1e-9, self.step_ms / 1e3):.0f} tok/s")


class Trainer:
    def __init__(self, model_cfg, train_cfg: TrainConfig, weights, rank: int = 0, world: int = 1, device="cuda",
                 group=None):
        self.cfg = train_cfg
        self.rank, self.world, self.group = rank, world, group
        self.device = torch.device(device)
        self.model = TrainableDecoder(model_cfg, weights, rank, world, self.device, group,
                                      activation_checkpointing=train_cfg.activation_checkpointing,
                                      param_dtype=getattr(torch, train_cfg.param_dtype))
        self.step_num = 0
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._coef = torch.ones(1, dtype=torch.float32, device=self.device)

    # -- one optimizer step ------------------------------------------------------
    def step(self, batch: torch.Tensor) -> StepMetrics:
        """``batch``: this rank's [B_local, S + 1] token ids (inputs + shifted targets)."""
        t0 = time.perf_counter()
        c = self.cfg
        batch = batch.to(self.device)
        ids, tgt = batch[:, :-1].contiguous(), batch[:, 1:].contiguous()
        B_local, S = ids.shape
        global_tokens = float(B_local * S * self.world)  # mean over the global batch
        total = torch.zeros((), dtype=torch.float32, device=self.device)
        mb = max(1, c.micro_batch)
        for s in range(0, B_local, mb):
            loss = self.model.loss(ids[s:s + mb], tgt[s:s + mb], denom=global_tokens)
            loss.backward()
            total += loss.detach()
        if self.world > 1:
            dist.all_reduce(total, group=self.group)
        gnorm = self._clip_coef()
        lr = c.lr_at(self.step_num)
        self.step_num += 1
        for g in self.model.groups:
            self._adamw(g, lr)
            g.grad.zero_()
        torch.cuda.synchronize(self.device) if self.device.type == "cuda" else None
        ms = (time.perf_counter() - t0) * 1e3
        return StepMetrics(self.step_num, float(total.item()), float(gnorm.item()), lr, int(global_tokens), ms)

    def _clip_coef(self) -> torch.Tensor:
        """Global L2 norm of the gradient shards; clip coefficient stays on the device."""
        self._sumsq.zero_()
        for g in self.model.groups:
            if g.grad.is_cuda:
                ops.ext().sumsq(g.grad, self._sumsq)
            else:
                self._sumsq += g.grad.float().pow(2).sum()
        if self.world > 1:
            dist.all_reduce(self._sumsq, group=self.group)
        norm = self._sumsq.sqrt()
        if self.cfg.grad_clip and self.cfg.grad_clip > 0:
            torch.clamp(self.cfg.grad_clip / (norm + 1e-6), max=1.0, out=self._coef)
        else:
            self._coef.fill_(1.0)
        return norm

    def _adamw(self, g: FlatGroup, lr: float):
        c = self.cfg
        if g.master.is_cuda:
            ops.ext().adamw(g.master, g.grad, g.exp_avg, g.exp_avg_sq, g.param, lr, c.betas[0], c.betas[1], c.eps,
                            c.weight_decay, self.step_num, self._coef, 1.0)
            ops._count(1)
            return
        b1, b2 = c.betas
        gr = g.grad * self._coef
        g.exp_avg.mul_(b1).add_(gr, alpha=1 - b1)
        g.exp_avg_sq.mul_(b2).addcmul_(gr, gr, value=1 - b2)
        mh = g.exp_avg / (1 - b1 ** self.step_num)
        vh = g.exp_avg_sq / (1 - b2 ** self.step_num)
        g.master -= lr * (mh / (vh.sqrt() + c.eps) + c.weight_decay * g.master)
        g.param.copy_(g.master)

    # -- checkpoints -------------------------------------------------------------
    def save_checkpoint(self, directory: str):
        """Each rank writes its shards; rank 0 writes the index (world-size agnostic)."""
        os.makedirs(directory, exist_ok=True)
        tensors = {}
        for g in self.model.groups:
            tensors[f"{g.name}.master"] = g.master.cpu()
            tensors[f"{g.name}.exp_avg"] = g.exp_avg.cpu()
            tensors[f"{g.name}.exp_avg_sq"] = g.exp_avg_sq.cpu()
        save_file(tensors, os.path.join(directory, f"shard-{self.rank:05d}.safetensors"),
                  {"rank": self.rank, "world": self.world})
        if self.rank == 0:
            meta = {"world": self.world, "step": self.step_num, "train_config": asdict(self.cfg),
                    "groups": {g.name: {"numel": g.numel, "padded": g.padded} for g in self.model.groups}}
            with open(os.path.join(directory, "index.json"), "w") as f:
                json.dump(meta, f, indent=1)
        if self.world > 1:
            dist.barrier(group=self.group)

    def load_checkpoint(self, directory: str):
        """Load shards written at any world size and re-shard for this one."""
        with open(os.path.join(directory, "index.json")) as f:
            meta = json.load(f)
        old_w = meta["world"]
        ckpts = [Checkpoint(os.path.join(directory, f"shard-{r:05d}.safetensors")) for r in range(old_w)]
        for g in self.model.groups:
            for field_name in ("master", "exp_avg", "exp_avg_sq"):
                full = torch.cat([ck.get(f"{g.name}.{field_name}") for ck in ckpts])[:g.numel]
                shard = torch.zeros(g.shard_n, dtype=torch.float32)
                lo = g.rank * g.shard_n
                hi = min(g.numel, lo + g.shard_n)
                if hi > lo:
                    shard[:hi - lo] = full[lo:hi]
                getattr(g, field_name).copy_(shard.to(g.device))
            g.param.copy_(g.master)
        self.step_num = int(meta["step"])
        for ck in ckpts:
            ck.close()

    def export_hf(self, directory: str):
        """Consolidated HF-named safetensors (bf16) + config.json, from rank 0."""
        from ..weights.weight_map import WeightMap
        sd = self.model.hf_state_dict()
        if self.rank == 0:
            WeightMap({k: v.to(torch.bfloat16).cpu() for k, v in sd.items()}).save(directory)
            self.model.cfg.save(directory)
        if self.world > 1:
            dist.barrier(group=self.group)
