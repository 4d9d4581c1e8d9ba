"""``WeightMap``: name -> tensor store with strict draining and rank slicing.

Mirrors the reference's weight_map / WeightLoader contract
(rlx-models-core src/weight_map.rs:88 `WeightMap`, :150 `drain_loader`,
:323 `take_transposed`, :397 `from_safetensors_dir_selected`;
src/weight_loader.rs:614-747 the `WeightLoader` trait): builders ``take``
tensors by HF name; whatever is left at the end is reported (strict mode
raises, like `AllF32StrictUnused`). B200 differences: tensors keep their
checkpoint dtype (no f32 blow-up), stay lazily mmap'd until taken, and
``take_shard`` slices a tensor for a tensor/expert-parallel rank at read time.
"""
from __future__ import annotations

import os
from typing import Callable, Iterable

import torch

from .safetensors_io import Checkpoint, save_sharded


class MissingWeight(KeyError):
    pass


class UnusedWeights(RuntimeError):
    pass


class WeightMap:
    def __init__(self, source: Checkpoint | dict[str, torch.Tensor] | None = None,
                 aliases: dict[str, str] | None = None):
        self._ckpt: Checkpoint | None = None
        self._dict: dict[str, torch.Tensor] = {}
        if isinstance(source, Checkpoint):
            self._ckpt = source
            self._names = set(source.keys())
        elif isinstance(source, dict):
            self._dict = dict(source)
            self._names = set(self._dict)
        else:
            self._names = set()
        self._taken: set[str] = set()
        self.aliases = dict(aliases or {})

    # -- construction ---------------------------------------------------------
    @classmethod
    def from_dir(cls, path: str, selected: Callable[[str], bool] | None = None) -> "WeightMap":
        wm = cls(Checkpoint(path))
        if selected is not None:
            wm._names = {n for n in wm._names if selected(n)}
        return wm

    @classmethod
    def from_file(cls, path: str) -> "WeightMap":
        return cls(Checkpoint(path))

    # -- queries --------------------------------------------------------------
    def _resolve(self, name: str) -> str:
        if name in self._names:
            return name
        alt = self.aliases.get(name)
        if alt is not None and alt in self._names:
            return alt
        raise MissingWeight(name)

    def __contains__(self, name: str) -> bool:
        try:
            self._resolve(name)
            return True
        except MissingWeight:
            return False

    def keys(self) -> list[str]:
        return sorted(self._names)

    def remaining_keys(self) -> list[str]:
        return sorted(self._names - self._taken)

    def peek(self, name: str) -> torch.Tensor:
        n = self._resolve(name)
        return self._ckpt.get(n) if self._ckpt is not None else self._dict[n]

    def shape(self, name: str) -> list[int]:
        n = self._resolve(name)
        if self._ckpt is not None:
            return self._ckpt.info(n)[1]
        return list(self._dict[n].shape)

    # -- taking ---------------------------------------------------------------
    def take(self, name: str, dtype: torch.dtype | None = None, device=None) -> torch.Tensor:
        t = self.peek(name)
        self._taken.add(self._resolve(name))
        if dtype is not None or device is not None:
            t = t.to(device=device if device is not None else t.device, dtype=dtype or t.dtype)
        return t

    def take_optional(self, name: str, **kw) -> torch.Tensor | None:
        return self.take(name, **kw) if name in self else None

    def take_transposed(self, name: str, **kw) -> torch.Tensor:
        return self.take(name, **kw).t().contiguous()

    def take_shard(self, name: str, dim: int, rank: int, world: int, **kw) -> torch.Tensor:
        """Contiguous 1/world slice along ``dim`` (tensor-parallel / expert-parallel rank)."""
        t = self.peek(name)
        self._taken.add(self._resolve(name))
        n = t.shape[dim]
        assert n % world == 0, f"{name}: dim {dim} ({n}) not divisible by {world}"
        step = n // world
        t = t.narrow(dim, rank * step, step)
        dtype, device = kw.get("dtype"), kw.get("device")
        if dtype is not None or device is not None:
            t = t.to(device=device if device is not None else t.device, dtype=dtype or t.dtype)
        return t.contiguous()

    def finish(self, strict: bool = True, ignore: Iterable[str] = ()) -> list[str]:
        """Report (or, strict, reject) tensors no builder consumed."""
        ign = tuple(ignore)
        left = [n for n in self.remaining_keys() if not any(n.startswith(p) for p in ign)]
        if strict and left:
            raise UnusedWeights(f"{len(left)} unused tensors, e.g. {left[:5]}")
        return left

    # -- misc -----------------------------------------------------------------
    def merge_add(self, name: str, delta: torch.Tensor):
        """In-memory ``W += delta`` (LoRA merge into a dict-backed map)."""
        n = self._resolve(name)
        base = self.peek(n)
        self._dict[n] = (base.float() + delta.float()).to(base.dtype)
        self._names.add(n)

    def to_dict(self) -> dict[str, torch.Tensor]:
        return {n: self.peek(n) for n in self.keys()}

    def save(self, directory: str, max_shard_bytes: int = 4 << 30):
        return save_sharded(self.to_dict(), directory, max_shard_bytes)


def checkpoint_exists(path: str) -> bool:
    if os.path.isdir(path):
        return any(f.endswith(".safetensors") for f in os.listdir(path))
    return path.endswith(".safetensors") and os.path.exists(path)
