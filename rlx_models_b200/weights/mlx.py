"""MLX-format quantised safetensors checkpoints.

MLX stores an affine group-quantised linear weight W [out, in] as three
tensors: ``<name>.weight`` uint32 [out, in * bits / 32] with the codes of
consecutive input columns packed from the least significant bits up,
``<name>.scales`` and ``<name>.biases`` [out, in / group_size] (fp16 / bf16),
and config.json carries ``"quantization": {"group_size": g, "bits": b}``
(optionally per-module overrides). The value of code q in group j is
``scales[:, j] * q + biases[:, j]``. Embeddings are quantised the same way.

``MLXWeights`` presents such a checkpoint to the model builders under the HF
names with dense tensors (dequantised on the target device), so MLX-converted
models load into the same kernels as bf16 checkpoints.

Reference: the reference's ``MlxLoader`` and ``take_packed_mlx``
(rlx-models-core src/weight_loader.rs:935) read the same layout through the
external rlx-mlx-io crate.
"""
from __future__ import annotations

import json
import os

import torch

from .weight_map import WeightMap


def unpack_codes(wq: torch.Tensor, bits: int) -> torch.Tensor:
    """uint32 [rows, in * bits / 32] (stored as int32 / uint32) -> int32 codes [rows, in]."""
    if bits not in (2, 4, 8):
        raise NotImplementedError(f"MLX {bits}-bit codes (2, 4 and 8 are supported)")
    per = 32 // bits
    w = wq.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(per, device=w.device, dtype=torch.int64) * bits
    q = (w.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)
    return q.reshape(w.shape[0], -1).to(torch.int32)


def dequantize(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int, group_size: int,
               dtype: torch.dtype = torch.float32) -> torch.Tensor:
    q = unpack_codes(wq, bits).float()
    rows, cols = q.shape
    g = q.view(rows, cols // group_size, group_size)
    w = g * scales.float().unsqueeze(-1) + biases.float().unsqueeze(-1)
    return w.view(rows, cols).to(dtype)


def quantize(w: torch.Tensor, bits: int = 4, group_size: int = 64):
    """Affine min/max group quantisation in the MLX layout -> (uint32-packed
    codes as int32, scales, biases) with fp16 scales and biases."""
    rows, cols = w.shape
    g = w.float().view(rows, cols // group_size, group_size)
    lo, hi = g.amin(-1), g.amax(-1)
    levels = (1 << bits) - 1
    scale = ((hi - lo) / levels).clamp_min(1e-8)
    q = ((g - lo.unsqueeze(-1)) / scale.unsqueeze(-1)).round().clamp(0, levels).to(torch.int64)
    q = q.view(rows, cols)
    per = 32 // bits
    shifts = torch.arange(per, dtype=torch.int64) * bits
    packed = (q.view(rows, cols // per, per) << shifts).sum(-1)
    packed = torch.where(packed >= 2 ** 31, packed - 2 ** 32, packed).to(torch.int32)
    return packed, scale.half(), lo.half()


class MLXWeights:
    """HF-named dense view of an MLX quantised checkpoint directory."""

    def __init__(self, path: str, device=None, dtype: torch.dtype = torch.bfloat16):
        self.wm = WeightMap.from_dir(path)
        with open(os.path.join(path, "config.json")) as f:
            cfg = json.load(f)
        q = cfg.get("quantization") or cfg.get("quantization_config") or {}
        self.bits = int(q.get("bits", 4))
        self.group_size = int(q.get("group_size", 64))
        self.overrides = {k: v for k, v in q.items() if isinstance(v, dict)}
        self.device, self.dtype = device, dtype
        names = set(self.wm.keys())
        self._quant = {n for n in names if n.endswith(".weight") and n[:-len(".weight")] + ".scales" in names}
        self._names = [n for n in names if not (n.endswith(".scales") or n.endswith(".biases"))
                       or n[:-len(".scales")] + ".weight" not in names]

    @staticmethod
    def is_mlx_dir(path: str) -> bool:
        try:
            with open(os.path.join(path, "config.json")) as f:
                cfg = json.load(f)
        except OSError:
            return False
        q = cfg.get("quantization")
        return isinstance(q, dict) and "bits" in q and "group_size" in q

    def keys(self):
        return list(self._names)

    def __contains__(self, name):
        return name in self._names

    def __getitem__(self, name):
        return self.take(name)

    def take(self, name: str) -> torch.Tensor:
        if name not in self._quant:
            t = self.wm.take(name)
            return t if self.device is None else t.to(self.device)
        base = name[:-len(".weight")]
        ov = self.overrides.get(base, {})
        bits, gs = int(ov.get("bits", self.bits)), int(ov.get("group_size", self.group_size))
        dev = self.device or "cpu"
        wq = self.wm.take(name).to(dev)
        sc = self.wm.take(base + ".scales").to(dev)
        bi = self.wm.take(base + ".biases").to(dev)
        return dequantize(wq, sc, bi, bits, gs, self.dtype)


def save_mlx(directory: str, tensors: dict[str, torch.Tensor], config: dict, bits: int = 4, group_size: int = 64,
             skip=("norm", "bias")):
    """Write HF-named tensors as an MLX quantised checkpoint (2-D weights
    quantised; norms, biases and 1-D tensors kept)."""
    os.makedirs(directory, exist_ok=True)
    out = {}
    for n, t in tensors.items():
        if t.dim() == 2 and n.endswith(".weight") and not any(s in n for s in skip) and t.shape[1] % group_size == 0:
            wq, sc, bi = quantize(t, bits, group_size)
            base = n[:-len(".weight")]
            out[n], out[base + ".scales"], out[base + ".biases"] = wq, sc, bi
        else:
            out[n] = t
    WeightMap(out).save(directory)
    cfg = dict(config)
    cfg["quantization"] = {"group_size": group_size, "bits": bits}
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return directory
