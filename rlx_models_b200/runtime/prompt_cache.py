"""Prompt-cache persistence: save a prompt's cached KV blocks to a file and
load them into another engine (another process, a later run).

The engine's prefix cache keys every full 16-token KV block by a chained hash
of its tokens. ``save_prompt`` writes the cached blocks of a prompt's longest
full-block prefix (K and V pages of every layer) to a ``.safetensors`` file
together with the prompt tokens and a model fingerprint; ``load_prompt``
verifies the fingerprint, allocates blocks in the scheduler, registers their
hashes as free-but-cached (so the next request that starts with these tokens
reuses them instead of recomputing) and copies the pages in. A file from a
different model (config, KV layout or weights) is refused and ``load_prompt``
returns 0, like the reference's stale-cache check.

Reference: rlx-models-core src/prompt_cache.rs:201-240 (`save_entry` /
`load_entry`: magic, fingerprint, tokens, per-layer K/V).
"""
from __future__ import annotations

import dataclasses
import hashlib
import json

import torch

from ..weights.safetensors_io import SafetensorsFile, save_file
from .kv_cache import BLOCK_SIZE

FORMAT = "rlx_models_b200.prompt_cache/1"


def model_fingerprint(model, kv) -> str:
    """Hex digest of the model configuration, the KV layout and a sample of the
    weights (the first 4096 values of the embedding and of the first layer's
    projection): two models that would fill the cache differently differ here."""
    h = hashlib.sha256()
    cfg = model.cfg
    h.update(json.dumps(dataclasses.asdict(cfg) if dataclasses.is_dataclass(cfg) else str(cfg), sort_keys=True,
                        default=str).encode())
    h.update(json.dumps([list(kv.k.shape), str(kv.k.dtype), BLOCK_SIZE,
                         getattr(model, "tp_rank", 0), getattr(model, "tp_size", 1)]).encode())
    samples = []
    if getattr(model, "embed", None) is not None:
        samples.append(model.embed.reshape(-1)[:4096])
    layers = getattr(model, "layers", None)
    if layers and getattr(layers[0], "wqkv", None) is not None:
        samples.append(layers[0].wqkv.reshape(-1)[:4096])
    for t in samples:
        h.update(t.detach().float().cpu().numpy().tobytes())
    return h.hexdigest()


def save_prompt(engine, path: str, tokens: list[int]) -> int:
    """Write the cached KV of ``tokens``' longest cached full-block prefix;
    returns the number of tokens saved (0: nothing cached)."""
    tokens = [int(t) for t in tokens]
    blocks = engine.sched.prefix_blocks(tokens)
    n = len(blocks)
    kv = engine.kv
    idx = torch.tensor(blocks, dtype=torch.long, device=kv.k.device)
    tensors = {"k": kv.k.index_select(1, idx).cpu() if n else torch.empty(0),
               "v": kv.v.index_select(1, idx).cpu() if n else torch.empty(0),
               "tokens": torch.tensor(tokens[:n * BLOCK_SIZE], dtype=torch.int32)}
    meta = {"format": FORMAT, "fingerprint": model_fingerprint(engine.model, kv), "blocks": str(n)}
    save_file(tensors, path, metadata=meta)
    return n * BLOCK_SIZE


def load_prompt(engine, path: str) -> int:
    """Restore a saved prompt prefix into ``engine``'s prefix cache; returns the
    number of tokens now cached (0 when the file belongs to another model or
    the engine runs without prefix caching)."""
    f = SafetensorsFile(path)
    try:
        meta = f.metadata
        if meta.get("format") != FORMAT or meta.get("fingerprint") != model_fingerprint(engine.model, engine.kv):
            return 0
        if not engine.cfg.prefix_caching:
            return 0
        tokens = f.get("tokens").tolist()
        blocks = engine.sched.import_prefix(tokens)
        kv = engine.kv
        k, v = f.get("k").clone(), f.get("v").clone()  # copies: the file's mapping closes below
        fill = [(i, b) for i, b in enumerate(blocks) if b >= 0]
        if fill:
            src = torch.tensor([i for i, _ in fill], dtype=torch.long)
            dst = torch.tensor([b for _, b in fill], dtype=torch.long, device=kv.k.device)
            kv.k.index_copy_(1, dst, k.index_select(1, src).to(kv.k.device))
            kv.v.index_copy_(1, dst, v.index_select(1, src).to(kv.v.device))
        return len(blocks) * BLOCK_SIZE
    finally:
        f.close()
