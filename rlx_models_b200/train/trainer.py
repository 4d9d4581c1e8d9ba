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
from ..utils.trace import nvtx
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
    lora_rank: int = 0             # > 0: freeze the base, train LoRA adapters of this rank
    lora_alpha: float = 32.0
    lora_targets: tuple = ("qkv", "o", "gate_up", "down")
    dora: bool = False
    # gradient reduce-scatter on CUDA: "push" adds every gradient element into
    # its owner's shard over NVLink (wgrad GEMM epilogue + push kernel, one
    # device barrier per step); "nccl" materialises full gradients and calls
    # reduce_scatter_tensor per group
    grad_reduce: str = "push"
    # quantisation-aware training: linear weights are fake-quantised to this
    # format in the forward pass (quant/calib.py FORMATS), gradients straight-through
    qat: str | None = None
    # "adamw", or "muon": orthogonalized Nesterov momentum for 2-D weights, AdamW for the rest (train/muon.py)
    optimizer: str = "adamw"
    muon_momentum: float = 0.95

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


class _Marks:
    """Phase boundaries of a step: CUDA events on the device, wall clock on CPU."""

    def __init__(self, device):
        self.cuda = device.type == "cuda"
        self.t = []

    def __call__(self):
        if self.cuda:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.t.append(e)
        else:
            self.t.append(time.perf_counter())

    def spans(self) -> list[float]:
        if self.cuda:
            return [a.elapsed_time(b) for a, b in zip(self.t, self.t[1:])]
        return [(b - a) * 1e3 for a, b in zip(self.t, self.t[1:])]


@dataclass
class StepMetrics:
    step: int
    loss: float
    grad_norm: float
    lr: float
    tokens: int
    step_ms: float
    compute_ms: float = 0.0   # forward + backward (device time on CUDA)
    comm_ms: float = 0.0      # gradient barrier / reductions after backward
    optim_ms: float = 0.0     # clip + AdamW

    @property
    def compute_fraction(self) -> float:
        tot = self.compute_ms + self.comm_ms + self.optim_ms
        return self.compute_ms / tot if tot > 0 else 0.0

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
        self.model.qat = train_cfg.qat
        self.lora = None
        if train_cfg.lora_rank > 0:
            from .lora import LoraAdapters
            self.lora = LoraAdapters(self.model, train_cfg.lora_rank, train_cfg.lora_alpha, train_cfg.lora_targets,
                                     train_cfg.dora, group=group, world=world)
            self.model.lora = self.lora
        self.push = None
        if train_cfg.grad_reduce == "push" and self.device.type == "cuda" and self.lora is None:
            from .fsdp import GradPush
            self.push = GradPush(self.model.groups, rank, world, self.device, group)
        self.step_num = 0
        self._sumsq = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._coef = torch.ones(1, dtype=torch.float32, device=self.device)

    @property
    def all_groups(self) -> list[FlatGroup]:
        return self.model.groups + ([self.lora.group_flat] if self.lora is not None else [])

    @property
    def opt_groups(self) -> list[FlatGroup]:
        """Groups the optimizer updates: the adapters when fine-tuning with LoRA."""
        return [self.lora.group_flat] if self.lora is not None else self.model.groups

    # -- one optimizer step ------------------------------------------------------
    def step(self, batch) -> StepMetrics:
        """``batch``: this rank's [B_local, S + 1] token ids (inputs + shifted
        targets), or a pair (ids [B, S], targets [B, S]) whose negative targets
        are ignored (prompt masking, padding)."""
        t0 = time.perf_counter()
        c = self.cfg
        if isinstance(batch, (tuple, list)):
            # valid targets counted where the batch lives (no device round trip for host batches)
            n_local = float((batch[1] >= 0).sum())
            ids, tgt = batch[0].to(self.device), batch[1].to(self.device)
        else:
            n_local = float((batch[:, 1:] >= 0).sum())
            batch = batch.to(self.device)
            ids, tgt = batch[:, :-1].contiguous(), batch[:, 1:].contiguous()
        B_local, S = ids.shape
        n_valid = torch.tensor([n_local], device=self.device)
        if self.world > 1:
            dist.all_reduce(n_valid, group=self.group)
        global_tokens = max(1.0, float(n_valid))  # mean over the global batch's valid targets
        total = torch.zeros((), dtype=torch.float32, device=self.device)
        mb = max(1, c.micro_batch)
        mark = _Marks(self.device)
        mark()
        with nvtx("train.forward_backward"):
            for s in range(0, B_local, mb):
                loss = self.model.loss(ids[s:s + mb], tgt[s:s + mb], denom=global_tokens)
                loss.backward()
                total += loss.detach()
        mark()
        with nvtx("train.reduce"):
            if self.push is not None:
                self.push.barrier()  # every rank's gradient pushes of this step have landed
            if self.world > 1:
                dist.all_reduce(total, group=self.group)
            if self.lora is not None:
                self.lora.allreduce_grad()
        mark()
        with nvtx("train.optimizer"):
            gnorm = self._clip_coef()
            lr = c.lr_at(self.step_num)
            self.step_num += 1
            for g in self.opt_groups:
                self._adamw(g, lr)
                g.grad.zero_()
        mark()
        torch.cuda.synchronize(self.device) if self.device.type == "cuda" else None
        ms = (time.perf_counter() - t0) * 1e3
        fb, red, opt = mark.spans()
        return StepMetrics(self.step_num, float(total.item()), float(gnorm.item()), lr, int(global_tokens), ms,
                           fb, red, opt)

    def dpo_step(self, chosen, rejected, beta: float = 0.1, ref_logps=None) -> StepMetrics:
        """One DPO optimizer step on preference pairs ((ids, targets) each, this
        rank's rows). Reference log-probs default to the frozen base model
        (adapters off) when training LoRA, else must be given."""
        from .losses import dpo_loss, sequence_logprob
        t0 = time.perf_counter()
        c = self.cfg
        (ci, ct), (ri, rt) = [(x.to(self.device), y.to(self.device)) for x, y in (chosen, rejected)]
        if ref_logps is None:
            assert self.lora is not None, "ref_logps are required when the full model is trained"
            with torch.no_grad():
                saved, self.model.lora = self.model.lora, None
                ref_c, ref_r = sequence_logprob(self.model, ci, ct), sequence_logprob(self.model, ri, rt)
                self.model.lora = saved
        else:
            ref_c, ref_r = (t.to(self.device) for t in ref_logps)
        loss = dpo_loss(sequence_logprob(self.model, ci, ct), sequence_logprob(self.model, ri, rt), ref_c, ref_r,
                        beta) / self.world
        loss.backward()
        total = loss.detach()
        if self.push is not None:
            self.push.barrier()
        if self.world > 1:
            dist.all_reduce(total, group=self.group)
        if self.lora is not None:
            self.lora.allreduce_grad()
        gnorm = self._clip_coef()
        lr = c.lr_at(self.step_num)
        self.step_num += 1
        for g in self.opt_groups:
            self._adamw(g, lr)
            g.grad.zero_()
        ms = (time.perf_counter() - t0) * 1e3
        return StepMetrics(self.step_num, float(total.item()), float(gnorm.item()), lr, int(ci.numel() + ri.numel()), ms)

    def _clip_coef(self) -> torch.Tensor:
        """Global L2 norm of the gradient shards; clip coefficient stays on the device."""
        self._sumsq.zero_()
        for g in self.opt_groups:
            if g.grad.is_cuda:
                ops.ext().sumsq(g.grad, self._sumsq)
            else:
                self._sumsq += g.grad.float().pow(2).sum()
        if self.world > 1 and self.lora is None:  # adapter gradients are already all-reduced
            dist.all_reduce(self._sumsq, group=self.group)
        norm = self._sumsq.sqrt()
        if self.cfg.grad_clip and self.cfg.grad_clip > 0:
            torch.clamp(self.cfg.grad_clip / (norm + 1e-6), max=1.0, out=self._coef)
        else:
            self._coef.fill_(1.0)
        return norm

    def _adamw(self, g: FlatGroup, lr: float):
        c = self.cfg
        if c.optimizer == "muon" and self.lora is None:
            from .muon import muon_step
            muon_step(self, g, lr)
            return
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
        for g in self.all_groups:
            tensors[f"{g.name}.master"] = g.master.cpu()
            tensors[f"{g.name}.exp_avg"] = g.exp_avg.cpu()
            tensors[f"{g.name}.exp_avg_sq"] = g.exp_avg_sq.cpu()
        save_file(tensors, os.path.join(directory, f"shard-{self.rank:05d}.safetensors"),
                  {"rank": self.rank, "world": self.world})
        if self.rank == 0:
            meta = {"world": self.world, "step": self.step_num, "train_config": asdict(self.cfg),
                    "groups": {g.name: {"numel": g.numel, "padded": g.padded} for g in self.all_groups}}
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
        for g in self.all_groups:
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
        if self.lora is not None:  # fold the adapters into the exported weights
            from .model import split_fused
            fused = {}
            for (i, t), W in self.lora.merged().items():
                p = f"model.layers.{i}."
                name = {"qkv": p + "self_attn.qkv_proj.weight", "o": p + "self_attn.o_proj.weight",
                        "gate_up": p + "mlp.gate_up_proj.weight", "down": p + "mlp.down_proj.weight"}[t]
                fused[name] = W
            sd.update(split_fused(fused, self.model.cfg))
        if self.rank == 0:
            WeightMap({k: v.to(torch.bfloat16).cpu() for k, v in sd.items()}).save(directory)
            self.model.cfg.save(directory)
        if self.world > 1:
            dist.barrier(group=self.group)
