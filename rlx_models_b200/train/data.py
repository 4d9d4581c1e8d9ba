"""Datasets for fine-tuning: JSONL in, fixed-shape (ids, targets) batches out.

Accepted records (one JSON object per line):
  {"text": ...}                        causal LM on the whole text; texts are
                                       concatenated with EOS and cut into
                                       seq_len windows (packing)
  {"prompt": ..., "completion": ...}   loss on the completion only (prompt
                                       targets masked with -1), one example
                                       per row, right-padded
  {"input_ids": [...], "labels": [...]}  pre-tokenised (labels optional)
  {"prompt", "chosen", "rejected"}     preference pairs (``PreferencePairs``)
Batches are deterministic (seeded shuffle) and split across data-parallel
ranks by index.

Reference: rlx-tune src/dataset.rs (JSONL text / prompt-completion loading,
packing) and src/loss.rs (masked next-token loss, DPO).
"""
from __future__ import annotations

import json
import random

import torch


def read_jsonl(path: str) -> list[dict]:
    with open(path) as f:
        return [json.loads(ln) for ln in f if ln.strip()]


class SFTDataset:
    def __init__(self, records: list[dict], tokenizer, seq_len: int, eos_id: int | None = None):
        self.seq_len = seq_len
        eos = eos_id if eos_id is not None else getattr(tokenizer, "eos_token_id", None)
        rows: list[tuple[list[int], list[int]]] = []
        stream: list[int] = []
        for r in records:
            if "input_ids" in r:
                ids = list(r["input_ids"])
                labels = list(r.get("labels", ids))
                rows.append(self._shift(ids, labels))
            elif "prompt" in r and "completion" in r:
                p = tokenizer.encode(r["prompt"])
                c = tokenizer.encode(r["completion"]) + ([eos] if eos is not None else [])
                ids = p + c
                labels = [-1] * len(p) + c
                rows.append(self._shift(ids, labels))
            elif "text" in r:
                stream += tokenizer.encode(r["text"]) + ([eos] if eos is not None else [])
        for s in range(0, len(stream) - 1, seq_len):
            chunk = stream[s:s + seq_len + 1]
            if len(chunk) < 2:
                break
            rows.append(self._shift(chunk, chunk))
        self.rows = rows

    def _shift(self, ids, labels):
        ids, labels = ids[:self.seq_len + 1], labels[:self.seq_len + 1]
        x, y = ids[:-1], labels[1:]
        pad = self.seq_len - len(x)
        return x + [0] * pad, y + [-1] * pad

    def __len__(self):
        return len(self.rows)

    def batches(self, batch: int, rank: int = 0, world: int = 1, seed: int = 0, epochs: int = 1000000):
        """Yield (ids, targets) int64 [batch, seq_len] for this rank (batch = per-rank size)."""
        n = len(self.rows)
        for ep in range(epochs):
            order = list(range(n))
            random.Random(seed + ep).shuffle(order)
            step = batch * world
            for s in range(0, n - step + 1, step):
                idx = order[s + rank * batch:s + (rank + 1) * batch]
                x = torch.tensor([self.rows[i][0] for i in idx], dtype=torch.int64)
                y = torch.tensor([self.rows[i][1] for i in idx], dtype=torch.int64)
                yield x, y


class PreferencePairs:
    """{"prompt", "chosen", "rejected"} -> (ids, targets) for chosen and rejected (prompt masked)."""

    def __init__(self, records, tokenizer, seq_len: int):
        self.pairs = []
        ds = SFTDataset([], tokenizer, seq_len)
        for r in records:
            p = tokenizer.encode(r["prompt"])
            ch = p + tokenizer.encode(r["chosen"])
            rj = p + tokenizer.encode(r["rejected"])
            mask = lambda ids: [-1] * len(p) + ids[len(p):]
            self.pairs.append((ds._shift(ch, mask(ch)), ds._shift(rj, mask(rj))))

    def batch(self, idx: list[int]):
        t = lambda k, j: torch.tensor([self.pairs[i][k][j] for i in idx], dtype=torch.int64)
        return (t(0, 0), t(0, 1)), (t(1, 0), t(1, 1))


def train_from_jsonl(a) -> int:
    """CLI: fine-tune a model on a JSONL file (single process or torchrun ranks)."""
    import os

    import torch.distributed as dist

    from ..api import resolve_model_path
    from ..config import DecoderConfig, preset
    from ..registry import RandomWeights
    from ..tokenizer import load_tokenizer
    from ..weights.weight_map import WeightMap
    from .trainer import TrainConfig, Trainer

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0))) if torch.cuda.is_available() else \
        torch.device("cpu")
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl" if dev.type == "cuda" else "gloo", timeout=timedelta(seconds=300))
    path = resolve_model_path(a.model)
    if path:
        cfg, weights = DecoderConfig.from_file(path), WeightMap.from_dir(path)
    else:
        cfg = preset(a.model)
        weights = RandomWeights(cfg, 0, dev)
    tok = load_tokenizer(path)
    ds = SFTDataset(read_jsonl(a.data), tok, a.seq_len)
    base = dict(lr=a.lr, total_steps=a.steps, micro_batch=max(1, a.batch // 4), lora_rank=a.lora_rank,
                param_dtype="bfloat16" if dev.type == "cuda" else "float32")
    rc = getattr(a, "run_config", None)
    if rc is not None and rc.train:
        # the config file's train section over the parser defaults; explicit flags win
        dflt = getattr(a, "_defaults", {})
        explicit = {f: getattr(a, d) for d, f in (("lr", "lr"), ("steps", "total_steps"), ("lora_rank", "lora_rank"))
                    if getattr(a, d) != dflt.get(d)}
        tcfg = rc.train_config(**{**{k: v for k, v in base.items() if k not in rc.train}, **explicit})
    else:
        tcfg = TrainConfig(**base)
    tr = Trainer(cfg, tcfg, weights, rank=rank, world=world, device=dev)
    it = ds.batches(a.batch, rank, world)
    for _ in range(a.steps):
        m = tr.step(next(it))
        if rank == 0:
            print(m, flush=True)
    if a.out:
        tr.export_hf(a.out)
    if world > 1:
        dist.destroy_process_group()
    return 0
