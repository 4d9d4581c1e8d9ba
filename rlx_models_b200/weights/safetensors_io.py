"""Safetensors reading (zero-copy mmap) and writing, single file or sharded.

Format: 8-byte little-endian header length N, N bytes of JSON
``{name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}}``,
then the raw little-endian tensor bytes. Sharded checkpoints carry a
``model.safetensors.index.json`` with ``{"weight_map": {name: file}}``.

Reference: rlx-models-core src/safetensors_checkpoint.rs:33-409
(`SafetensorsCheckpoint`, per-tensor raw / f32 / row-range reads,
`load_selected`). Unlike the reference, tensors keep their stored dtype (bf16
stays bf16) and row-range reads return views, which is what rank-sliced
TP/EP/FSDP loading needs.
"""
from __future__ import annotations

import json
import mmap
import os
import struct
from typing import Iterable

import torch

DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2,
}
DTYPE_NAMES = {v: k for k, v in DTYPES.items()}


class SafetensorsFile:
    """One mmap'd ``.safetensors`` file. ``get(name)`` returns a CPU view."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        n = struct.unpack("<Q", self._f.read(8))[0]
        self.header = json.loads(self._f.read(n))
        self.metadata = self.header.pop("__metadata__", {}) or {}
        self._base = 8 + n
        size = os.fstat(self._f.fileno()).st_size
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ) if size > 0 else None

    def keys(self) -> list[str]:
        return list(self.header.keys())

    def info(self, name: str) -> tuple[torch.dtype, list[int]]:
        h = self.header[name]
        return DTYPES[h["dtype"]], list(h["shape"])

    def get(self, name: str) -> torch.Tensor:
        h = self.header[name]
        dt = DTYPES[h["dtype"]]
        b, e = h["data_offsets"]
        shape = list(h["shape"])
        if e == b:
            return torch.empty(shape, dtype=dt)
        buf = memoryview(self._mm)[self._base + b:self._base + e]
        import warnings
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")  # read-only mmap: consumers copy before writing
            t = torch.frombuffer(buf, dtype=dt)
        return t.reshape(shape)

    def get_rows(self, name: str, start: int, stop: int) -> torch.Tensor:
        """Rows [start, stop) of dim 0 without touching the rest of the tensor."""
        return self.get(name)[start:stop]

    def close(self):
        if self._mm is not None:
            self._mm.close()
        self._f.close()


class Checkpoint:
    """A model directory (or file): one or more safetensors shards + index."""

    def __init__(self, path: str):
        self.path = path
        self.files: dict[str, SafetensorsFile] = {}
        self.where: dict[str, str] = {}
        if os.path.isdir(path):
            idx = os.path.join(path, "model.safetensors.index.json")
            if os.path.exists(idx):
                with open(idx) as f:
                    wm = json.load(f)["weight_map"]
                for name, fn in wm.items():
                    self.where[name] = os.path.join(path, fn)
            else:
                for fn in sorted(os.listdir(path)):
                    if fn.endswith(".safetensors"):
                        full = os.path.join(path, fn)
                        for k in self._file(full).keys():
                            self.where[k] = full
        else:
            for k in self._file(path).keys():
                self.where[k] = path

    def _file(self, fn: str) -> SafetensorsFile:
        f = self.files.get(fn)
        if f is None:
            f = SafetensorsFile(fn)
            self.files[fn] = f
        return f

    def keys(self) -> list[str]:
        return list(self.where.keys())

    def __contains__(self, name: str) -> bool:
        return name in self.where

    def get(self, name: str) -> torch.Tensor:
        return self._file(self.where[name]).get(name)

    def info(self, name: str):
        return self._file(self.where[name]).info(name)

    def load_selected(self, names: Iterable[str]) -> dict[str, torch.Tensor]:
        return {n: self.get(n) for n in names}

    def close(self):
        for f in self.files.values():
            f.close()
        self.files.clear()


def save_file(tensors: dict[str, torch.Tensor], path: str, metadata: dict[str, str] | None = None):
    """Write a single safetensors file (tensors are made contiguous on CPU)."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    off = 0
    items = []
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": DTYPE_NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + nbytes]}
        items.append(t)
        off += nbytes
    hb = json.dumps(header, separators=(",", ":")).encode()
    pad = (8 - len(hb) % 8) % 8
    hb += b" " * pad
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for t in items:
            if t.numel():
                flat = t.reshape(-1)  # 0-dim scalars too (a byte view needs at least one dim)
                f.write(flat.view(torch.uint8).numpy().tobytes() if t.dtype != torch.uint8 else flat.numpy().tobytes())
    os.replace(tmp, path)


def save_sharded(tensors: dict[str, torch.Tensor], directory: str, max_shard_bytes: int = 4 << 30,
                 metadata: dict[str, str] | None = None) -> list[str]:
    """Write ``model-0000i-of-0000n.safetensors`` shards plus the index json."""
    os.makedirs(directory, exist_ok=True)
    shards: list[dict[str, torch.Tensor]] = [{}]
    size = 0
    for name in sorted(tensors):
        t = tensors[name]
        nb = t.numel() * t.element_size()
        if shards[-1] and size + nb > max_shard_bytes:
            shards.append({})
            size = 0
        shards[-1][name] = t
        size += nb
    n = len(shards)
    files = []
    weight_map = {}
    total = 0
    for i, sh in enumerate(shards):
        fn = "model.safetensors" if n == 1 else f"model-{i + 1:05d}-of-{n:05d}.safetensors"
        save_file(sh, os.path.join(directory, fn), metadata)
        files.append(fn)
        for k, t in sh.items():
            weight_map[k] = fn
            total += t.numel() * t.element_size()
    if n > 1:
        with open(os.path.join(directory, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=1)
    return files
