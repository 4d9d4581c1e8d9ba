"""GGUF (v2/v3) checkpoints: reader, writer, block dequantisation, HF names.

A GGUF file is a header (magic ``GGUF``, version, tensor count, metadata
count), typed metadata key/values, tensor descriptors (name, dims with the
fastest-varying first, ggml type, offset) and an aligned data section. Tensors
are row-major; quantised types store each row as blocks along the innermost
dimension. This module reads such files lazily (numpy memmap), writes them
(tests, the quantisation tool's GGUF sink), dequantises every ggml block
format used by llama-family checkpoints - legacy Q4_0/Q4_1/Q5_0/Q5_1/Q8_0,
the K-quants Q2_K..Q6_K/Q8_K, F16/BF16/F32 - into torch tensors, maps GGUF
tensor names to the HF names the model builders take, and reads a
:class:`DecoderConfig` out of the metadata.

The block layouts and dequantisation formulas are those of the GGUF format
(they define the file's meaning, so any reader must match them); the code is
a vectorised torch restatement over whole tensors. ``ops.gguf_dequant`` runs
the same formulas as a CUDA kernel on device-resident blocks.

Reference: the reference reads GGUF through the external rlx-gguf crate via
``GgufLoader`` (rlx-models-core src/weight_loader.rs:1237), with HF <-> GGUF
name translation (`hf_to_gguf_name` :73, `gguf_to_hf_name` :116) and the ggml
type table (`ggml_type_to_quant_scheme` :497-554).
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass

import numpy as np
import torch

# ggml type id -> (name, elements per block, bytes per block)
GGML_TYPES: dict[int, tuple[str, int, int]] = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22),
    7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 36), 10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110),
    12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 15: ("Q8_K", 256, 292),
    24: ("I8", 1, 1), 25: ("I16", 1, 2), 26: ("I32", 1, 4), 27: ("I64", 1, 8), 28: ("F64", 1, 8),
    30: ("BF16", 1, 2),
}
TYPE_ID = {v[0]: k for k, v in GGML_TYPES.items()}

# metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}


@dataclass
class TensorInfo:
    name: str
    shape: tuple[int, ...]  # torch order (outermost first)
    ggml_type: int
    offset: int  # absolute file offset of the data

    @property
    def type_name(self) -> str:
        return GGML_TYPES[self.ggml_type][0]

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    @property
    def nbytes(self) -> int:
        _, be, bb = GGML_TYPES[self.ggml_type]
        return self.numel // be * bb


class GGUFReader:
    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._pos = 0
        if self._read(4) != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        self.version = self._unpack("<I")
        if self.version not in (2, 3):
            raise ValueError(f"{path}: unsupported GGUF version {self.version}")
        n_tensors = self._unpack("<Q")
        n_kv = self._unpack("<Q")
        self.metadata: dict = {}
        for _ in range(n_kv):
            key = self._string()
            self.metadata[key] = self._value(self._unpack("<I"))
        infos = []
        for _ in range(n_tensors):
            name = self._string()
            nd = self._unpack("<I")
            dims = [self._unpack("<Q") for _ in range(nd)]
            t = self._unpack("<I")
            off = self._unpack("<Q")
            if t not in GGML_TYPES:
                raise ValueError(f"{path}: tensor {name} has unsupported ggml type {t}")
            infos.append((name, tuple(reversed(dims)), t, off))
        align = int(self.metadata.get("general.alignment", 32))
        data_start = (self._pos + align - 1) // align * align
        self.tensors: dict[str, TensorInfo] = {n: TensorInfo(n, s, t, data_start + o) for n, s, t, o in infos}

    # -- low-level parsing -----------------------------------------------------
    def _read(self, n: int) -> bytes:
        b = self._mm[self._pos:self._pos + n]
        self._pos += n
        return b

    def _unpack(self, fmt: str):
        size = struct.calcsize(fmt)
        (v,) = struct.unpack_from(fmt, self._mm, self._pos)
        self._pos += size
        return v

    def _string(self) -> str:
        n = self._unpack("<Q")
        return self._read(n).decode("utf-8", errors="replace")

    def _value(self, vt: int):
        if vt in _SCALAR:
            return self._unpack(_SCALAR[vt])
        if vt == _STR:
            return self._string()
        if vt == _ARR:
            et = self._unpack("<I")
            n = self._unpack("<Q")
            if et in _SCALAR and et != _BOOL:
                dt = np.dtype(_SCALAR[et])
                arr = np.frombuffer(self._mm, dtype=dt, count=n, offset=self._pos).copy()
                self._pos += n * dt.itemsize
                return arr.tolist()
            return [self._value(et) for _ in range(n)]
        raise ValueError(f"unknown GGUF metadata type {vt}")

    # -- tensors ---------------------------------------------------------------
    def keys(self) -> list[str]:
        return list(self.tensors)

    def __contains__(self, name: str) -> bool:
        return name in self.tensors

    def raw(self, name: str) -> torch.Tensor:
        """The tensor's stored bytes as a uint8 tensor (no copy of the mapping)."""
        ti = self.tensors[name]
        arr = np.frombuffer(self._mm, dtype=np.uint8, count=ti.nbytes, offset=ti.offset)
        return torch.from_numpy(arr.copy())

    def get(self, name: str, dtype: torch.dtype = torch.float32, device=None) -> torch.Tensor:
        """Dequantised tensor in torch shape order. On a CUDA ``device`` the
        quantised blocks are copied over and expanded by the device kernel."""
        ti = self.tensors[name]
        raw = self.raw(name)
        if device is not None and torch.device(device).type == "cuda" and ti.type_name not in ("F32", "F64",
                                                                                                "I8", "I16",
                                                                                                "I32", "I64"):
            from .. import ops
            return ops.gguf_dequant(raw.to(device), ti.type_name, ti.shape, dtype)
        out = dequantize(raw, ti.type_name, ti.shape).to(dtype)
        return out if device is None else out.to(device)

    def close(self):
        self._mm.close()
        self._f.close()


# ---------------------------------------------------------------------------
# dequantisation (torch, vectorised over blocks)
# ---------------------------------------------------------------------------

def _f16(b: torch.Tensor) -> torch.Tensor:
    """[..., 2] uint8 -> [...] float32 (little-endian IEEE half)."""
    return b.contiguous().view(torch.float16).squeeze(-1).float()


def _nib(q: torch.Tensor):
    return (q & 0xF).to(torch.int32), (q >> 4).to(torch.int32)


def _k4_scale_min(s: torch.Tensor):
    """12 packed bytes -> 8 six-bit scales and 8 six-bit mins (Q4_K / Q5_K)."""
    s = s.to(torch.int32)
    sc = torch.empty(s.shape[0], 8, dtype=torch.int32, device=s.device)
    mn = torch.empty_like(sc)
    sc[:, :4] = s[:, 0:4] & 63
    mn[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 0xF) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc.float(), mn.float()


def _q3k_scales(s: torch.Tensor) -> torch.Tensor:
    """12 packed bytes -> 16 six-bit scales minus 32 (Q3_K)."""
    s = s.to(torch.int32)
    lo, hi = s[:, 0:8], s[:, 8:12]
    out = torch.empty(s.shape[0], 16, dtype=torch.int32, device=s.device)
    out[:, 0:4] = (lo[:, 0:4] & 0xF) | ((hi & 3) << 4)
    out[:, 4:8] = (lo[:, 4:8] & 0xF) | (((hi >> 2) & 3) << 4)
    out[:, 8:12] = (lo[:, 0:4] >> 4) | (((hi >> 4) & 3) << 4)
    out[:, 12:16] = (lo[:, 4:8] >> 4) | (((hi >> 6) & 3) << 4)
    return (out - 32).float()


def dequantize_blocks(raw: torch.Tensor, kind: str) -> torch.Tensor:
    """[nb * block_bytes] uint8 -> [nb * block_elems] float32."""
    tid = TYPE_ID[kind]
    _, be, bb = GGML_TYPES[tid]
    if kind == "F32":
        return raw.view(torch.float32).clone()
    if kind == "F16":
        return raw.view(torch.float16).float()
    if kind == "BF16":
        return raw.view(torch.bfloat16).float()
    if kind == "F64":
        return raw.view(torch.float64).float()
    if kind in ("I8", "I16", "I32", "I64"):
        return raw.view({"I8": torch.int8, "I16": torch.int16, "I32": torch.int32, "I64": torch.int64}[kind]).float()
    b = raw.view(-1, bb)
    nb = b.shape[0]
    if kind == "Q4_0":
        d = _f16(b[:, 0:2])
        lo, hi = _nib(b[:, 2:18])
        return ((torch.cat([lo, hi], 1) - 8).float() * d[:, None]).reshape(-1)
    if kind == "Q4_1":
        d, m = _f16(b[:, 0:2]), _f16(b[:, 2:4])
        lo, hi = _nib(b[:, 4:20])
        return (torch.cat([lo, hi], 1).float() * d[:, None] + m[:, None]).reshape(-1)
    if kind in ("Q5_0", "Q5_1"):
        off = 2 if kind == "Q5_0" else 4
        d = _f16(b[:, 0:2])
        qh = b[:, off:off + 4].to(torch.int64)
        qh = qh[:, 0] | (qh[:, 1] << 8) | (qh[:, 2] << 16) | (qh[:, 3] << 24)
        bits = ((qh[:, None] >> torch.arange(32, device=qh.device)) & 1).to(torch.int32)
        lo, hi = _nib(b[:, off + 4:off + 20])
        q = torch.cat([lo, hi], 1) | (bits << 4)
        if kind == "Q5_0":
            return ((q - 16).float() * d[:, None]).reshape(-1)
        m = _f16(b[:, 2:4])
        return (q.float() * d[:, None] + m[:, None]).reshape(-1)
    if kind == "Q8_0":
        d = _f16(b[:, 0:2])
        return (b[:, 2:34].view(torch.int8).float() * d[:, None]).reshape(-1)
    if kind == "Q8_1":
        d = _f16(b[:, 0:2])
        return (b[:, 4:36].view(torch.int8).float() * d[:, None]).reshape(-1)
    if kind == "Q8_K":
        d = b[:, 0:4].contiguous().view(torch.float32).squeeze(-1)
        return (b[:, 4:260].view(torch.int8).float() * d[:, None]).reshape(-1)
    if kind == "Q2_K":
        sc = b[:, 0:16].to(torch.int32)
        qs = b[:, 16:80].to(torch.int32).view(nb, 2, 32)
        d, dmin = _f16(b[:, 80:82]), _f16(b[:, 82:84])
        vals = torch.stack([(qs >> (2 * j)) & 3 for j in range(4)], 2)  # [nb, 2 (half), 4 (shift), 32]
        vals = vals.view(nb, 16, 16).float()  # sub-block order (half, shift, 16-group) = scale index
        dl = d[:, None] * (sc & 0xF).float()
        ml = dmin[:, None] * (sc >> 4).float()
        return (dl[:, :, None] * vals - ml[:, :, None]).reshape(-1)
    if kind == "Q3_K":
        hm = b[:, 0:32].to(torch.int32)
        qs = b[:, 32:96].to(torch.int32).view(nb, 2, 32)
        scales = _q3k_scales(b[:, 96:108])
        d = _f16(b[:, 108:110])
        q = torch.stack([(qs >> (2 * j)) & 3 for j in range(4)], 2)  # [nb, 2, 4, 32]
        mbit = torch.stack([torch.stack([(hm >> (4 * n + j)) & 1 for j in range(4)], 1) for n in range(2)], 1)
        vals = (q - 4 * (1 - mbit)).view(nb, 16, 16).float()
        return ((d[:, None] * scales)[:, :, None] * vals).reshape(-1)
    if kind in ("Q4_K", "Q5_K"):
        d, dmin = _f16(b[:, 0:2]), _f16(b[:, 2:4])
        sc, mn = _k4_scale_min(b[:, 4:16])
        if kind == "Q4_K":
            qs = b[:, 16:144].to(torch.int32).view(nb, 4, 32)
            vals = torch.stack([qs & 0xF, qs >> 4], 2)  # [nb, 4 (pair), 2, 32]
        else:
            qh = b[:, 16:48].to(torch.int32)
            qs = b[:, 48:176].to(torch.int32).view(nb, 4, 32)
            hb = torch.stack([torch.stack([(qh >> (2 * p)) & 1, (qh >> (2 * p + 1)) & 1], 1) for p in range(4)], 1)
            vals = torch.stack([qs & 0xF, qs >> 4], 2) + 16 * hb
        vals = vals.view(nb, 8, 32).float()
        return ((d[:, None] * sc)[:, :, None] * vals - (dmin[:, None] * mn)[:, :, None]).reshape(-1)
    if kind == "Q6_K":
        ql = b[:, 0:128].to(torch.int32).view(nb, 2, 64)
        qh = b[:, 128:192].to(torch.int32).view(nb, 2, 32)
        sc = b[:, 192:208].view(torch.int8).float().view(nb, 2, 8)
        d = _f16(b[:, 208:210])
        q1 = (ql[:, :, :32] & 0xF) | ((qh & 3) << 4)
        q2 = (ql[:, :, 32:] & 0xF) | (((qh >> 2) & 3) << 4)
        q3 = (ql[:, :, :32] >> 4) | (((qh >> 4) & 3) << 4)
        q4 = (ql[:, :, 32:] >> 4) | (((qh >> 6) & 3) << 4)
        q = (torch.stack([q1, q2, q3, q4], 2) - 32).float()  # [nb, 2, 4, 32]
        s = sc.view(nb, 2, 4, 2)  # scale index = 2 * quarter + (l >= 16)
        s = s.repeat_interleave(16, dim=3)  # [nb, 2, 4, 32]
        return (d[:, None, None, None] * s * q).reshape(-1)
    raise NotImplementedError(f"GGUF dequantisation of {kind}")


def dequantize(raw: torch.Tensor, kind: str, shape) -> torch.Tensor:
    return dequantize_blocks(raw.reshape(-1), kind).view(*shape)


# ---------------------------------------------------------------------------
# quantisation (for writing GGUF files)
# ---------------------------------------------------------------------------

def quantize(x: torch.Tensor, kind: str) -> torch.Tensor:
    """float tensor (rows a multiple of the block size) -> uint8 blocks."""
    x = x.float().contiguous()
    if kind == "F32":
        return x.view(-1).view(torch.uint8).clone()
    if kind == "F16":
        return x.half().view(-1).view(torch.uint8).clone()
    if kind == "BF16":
        return x.bfloat16().view(-1).view(torch.uint8).clone()
    v = x.view(-1, 32)
    if kind == "Q8_0":
        amax = v.abs().amax(1)
        d = (amax / 127).half()
        inv = torch.where(d.float() > 0, 1 / d.float(), torch.zeros_like(amax))
        q = (v * inv[:, None]).round().clamp(-127, 127).to(torch.int8)
        return torch.cat([d.view(-1, 1).view(torch.uint8), q.view(torch.uint8)], 1).reshape(-1)
    if kind == "Q4_0":
        idx = v.abs().argmax(1)
        mx = v.gather(1, idx[:, None]).squeeze(1)  # signed value of largest magnitude
        d = (mx / -8).half()
        inv = torch.where(d.float() != 0, 1 / d.float(), torch.zeros_like(mx))
        q = (v * inv[:, None] + 8.5).floor().clamp(0, 15).to(torch.uint8)
        packed = q[:, :16] | (q[:, 16:] << 4)
        return torch.cat([d.view(-1, 1).view(torch.uint8), packed], 1).reshape(-1)
    if kind == "Q6_K":
        sb = x.view(-1, 256)
        nb = sb.shape[0]
        sub = sb.view(nb, 16, 16)
        ls = sub.abs().amax(2) / 31  # per 16-element sub-block step, |q| <= 31
        d = (ls.amax(1) / 127).half()
        dinv = torch.where(d.float() > 0, 1 / d.float(), torch.zeros(nb, device=x.device))
        sc = (ls * dinv[:, None]).round().clamp(-128, 127).to(torch.int8)  # sub-block scales
        step = d.float()[:, None] * sc.float()
        q = torch.where(step[..., None] != 0, (sub / step[..., None]).round(), torch.zeros_like(sub))
        q = (q.clamp(-32, 31) + 32).to(torch.int32).view(nb, 2, 4, 32)  # [nb, half, quarter, 32]
        ql = torch.empty(nb, 2, 64, dtype=torch.int32, device=x.device)
        ql[:, :, :32] = (q[:, :, 0] & 0xF) | ((q[:, :, 2] & 0xF) << 4)
        ql[:, :, 32:] = (q[:, :, 1] & 0xF) | ((q[:, :, 3] & 0xF) << 4)
        qh = (q[:, :, 0] >> 4) | ((q[:, :, 1] >> 4) << 2) | ((q[:, :, 2] >> 4) << 4) | ((q[:, :, 3] >> 4) << 6)
        return torch.cat([ql.reshape(nb, 128).to(torch.uint8), qh.reshape(nb, 64).to(torch.uint8),
                          sc.view(torch.uint8), d.view(-1, 1).view(torch.uint8)], 1).reshape(-1)
    if kind == "Q4_K":
        sb = x.view(-1, 256)
        nb = sb.shape[0]
        sub = sb.view(nb, 8, 32)
        lo = sub.amin(2).clamp(max=0)
        hi = sub.amax(2)
        scale = (hi - lo) / 15  # per sub-block step, min = -lo
        d = (scale.amax(1) / 63).half()
        dmin = ((-lo).amax(1) / 63).half()
        dinv = torch.where(d.float() > 0, 1 / d.float(), torch.zeros(nb, device=x.device))
        minv = torch.where(dmin.float() > 0, 1 / dmin.float(), torch.zeros(nb, device=x.device))
        sc = (scale * dinv[:, None]).round().clamp(0, 63).to(torch.int32)
        mn = (-lo * minv[:, None]).round().clamp(0, 63).to(torch.int32)
        step = d.float()[:, None] * sc.float()
        off = dmin.float()[:, None] * mn.float()
        q = torch.where(step[..., None] > 0, ((sub + off[..., None]) / step[..., None]).round(),
                        torch.zeros_like(sub)).clamp(0, 15).to(torch.int32)  # [nb, 8, 32]
        packed = torch.empty(nb, 12, dtype=torch.int32, device=x.device)
        packed[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
        packed[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
        packed[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mn[:, 4:8] & 0xF) << 4)
        qv = q.view(nb, 4, 2, 32)
        qs = (qv[:, :, 0] | (qv[:, :, 1] << 4)).reshape(nb, 128)
        return torch.cat([d.view(-1, 1).view(torch.uint8), dmin.view(-1, 1).view(torch.uint8),
                          packed.to(torch.uint8), qs.to(torch.uint8)], 1).reshape(-1)
    raise NotImplementedError(f"GGUF quantisation to {kind}")


# ---------------------------------------------------------------------------
# writer
# ---------------------------------------------------------------------------

class GGUFWriter:
    def __init__(self, path: str, alignment: int = 32):
        self.path = path
        self.alignment = alignment
        self.metadata: dict[str, tuple[int, object]] = {}
        self.tensors: list[tuple[str, tuple[int, ...], int, bytes]] = []

    def add(self, key: str, value, vtype: int | None = None):
        if vtype is None:
            if isinstance(value, bool):
                vtype = _BOOL
            elif isinstance(value, int):
                vtype = _U32 if 0 <= value < 2 ** 32 else _I64
            elif isinstance(value, float):
                vtype = _F32
            elif isinstance(value, str):
                vtype = _STR
            elif isinstance(value, (list, tuple)):
                vtype = _ARR
            else:
                raise TypeError(key)
        self.metadata[key] = (vtype, value)

    def add_tensor(self, name: str, x: torch.Tensor, kind: str = "F32"):
        shape = tuple(int(d) for d in x.shape)
        self.tensors.append((name, shape, TYPE_ID[kind], quantize(x, kind).cpu().numpy().tobytes()))

    def add_raw(self, name: str, shape, kind: str, data: bytes):
        self.tensors.append((name, tuple(int(d) for d in shape), TYPE_ID[kind], bytes(data)))

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode()
        return struct.pack("<Q", len(b)) + b

    def _val(self, vt: int, v) -> bytes:
        if vt in _SCALAR:
            return struct.pack(_SCALAR[vt], v)
        if vt == _STR:
            return self._str(v)
        if vt == _ARR:
            items = list(v)
            et = _STR if items and isinstance(items[0], str) else (_F32 if items and isinstance(items[0], float)
                                                                    else _I32)
            return struct.pack("<IQ", et, len(items)) + b"".join(self._val(et, x) for x in items)
        raise ValueError(vt)

    def write(self):
        self.add("general.alignment", self.alignment)
        out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(self.tensors), len(self.metadata)))
        for k, (vt, v) in self.metadata.items():
            out += self._str(k) + struct.pack("<I", vt) + self._val(vt, v)
        off = 0
        offsets = []
        for name, shape, t, data in self.tensors:
            offsets.append(off)
            out += self._str(name) + struct.pack("<I", len(shape))
            out += b"".join(struct.pack("<Q", d) for d in reversed(shape))
            out += struct.pack("<IQ", t, off)
            off = (off + len(data) + self.alignment - 1) // self.alignment * self.alignment
        out += b"\0" * ((-len(out)) % self.alignment)
        for (name, shape, t, data), o in zip(self.tensors, offsets):
            out += data
            out += b"\0" * ((-len(data)) % self.alignment)
        with open(self.path, "wb") as f:
            f.write(out)


# ---------------------------------------------------------------------------
# names and config
# ---------------------------------------------------------------------------

_LAYER_MAP = {
    "attn_norm": "input_layernorm", "attn_q": "self_attn.q_proj", "attn_k": "self_attn.k_proj",
    "attn_v": "self_attn.v_proj", "attn_output": "self_attn.o_proj", "attn_q_norm": "self_attn.q_norm",
    "attn_k_norm": "self_attn.k_norm", "ffn_norm": "post_attention_layernorm", "ffn_gate": "mlp.gate_proj",
    "ffn_up": "mlp.up_proj", "ffn_down": "mlp.down_proj",
}
_GLOBAL_MAP = {"token_embd": "model.embed_tokens", "output_norm": "model.norm", "output": "lm_head"}
_HF_LAYER = {v: k for k, v in _LAYER_MAP.items()}
_HF_GLOBAL = {v: k for k, v in _GLOBAL_MAP.items()}


def gguf_to_hf_name(name: str) -> str | None:
    base, _, suffix = name.rpartition(".")
    if base in _GLOBAL_MAP:
        return f"{_GLOBAL_MAP[base]}.{suffix}"
    parts = base.split(".")
    if len(parts) == 3 and parts[0] == "blk" and parts[2] in _LAYER_MAP:
        return f"model.layers.{parts[1]}.{_LAYER_MAP[parts[2]]}.{suffix}"
    return None


def hf_to_gguf_name(name: str) -> str | None:
    base, _, suffix = name.rpartition(".")
    if base in _HF_GLOBAL:
        return f"{_HF_GLOBAL[base]}.{suffix}"
    if base.startswith("model.layers."):
        rest = base[len("model.layers."):]
        i, _, mod = rest.partition(".")
        if mod in _HF_LAYER:
            return f"blk.{i}.{_HF_LAYER[mod]}.{suffix}"
    return None


def permute_qk(w: torch.Tensor, n_head: int) -> torch.Tensor:
    """HF half-split rotary rows -> the interleaved-pair order GGUF ``llama``
    checkpoints store q/k projection rows in."""
    d = w.shape[0]
    return w.reshape(n_head, 2, d // n_head // 2, *w.shape[1:]).swapaxes(1, 2).reshape(w.shape)


def unpermute_qk(w: torch.Tensor, n_head: int) -> torch.Tensor:
    d = w.shape[0]
    return w.reshape(n_head, d // n_head // 2, 2, *w.shape[1:]).swapaxes(1, 2).reshape(w.shape)


_ARCH_MODEL_TYPE = {"llama": "llama", "mistral": "mistral", "qwen2": "qwen2", "qwen3": "qwen3"}


def config_from_metadata(md: dict, tensors: dict[str, TensorInfo]):
    from ..config import DecoderConfig
    arch = md.get("general.architecture", "llama")
    if arch not in _ARCH_MODEL_TYPE:
        raise NotImplementedError(f"GGUF architecture {arch!r}")

    def k(key, default=None):
        return md.get(f"{arch}.{key}", default)

    H = int(k("embedding_length"))
    nh = int(k("attention.head_count"))
    nkv = int(k("attention.head_count_kv", nh))
    emb = tensors["token_embd.weight"]
    vocab = len(md["tokenizer.ggml.tokens"]) if "tokenizer.ggml.tokens" in md else emb.shape[0]
    head_dim = int(k("attention.key_length", H // nh))
    return DecoderConfig(
        model_type=_ARCH_MODEL_TYPE[arch], vocab_size=vocab, hidden_size=H,
        intermediate_size=int(k("feed_forward_length")), num_hidden_layers=int(k("block_count")),
        num_attention_heads=nh, num_key_value_heads=nkv, head_dim=head_dim,
        rms_norm_eps=float(k("attention.layer_norm_rms_epsilon", 1e-6)), rope_theta=float(k("rope.freq_base", 1e4)),
        max_position_embeddings=int(k("context_length", 4096)),
        tie_word_embeddings="output.weight" not in tensors,
        qk_norm="blk.0.attn_q_norm.weight" in tensors,
        attention_bias="blk.0.attn_q.bias" in tensors)


class GGUFWeights:
    """HF-named, dequantised view of a GGUF checkpoint for the model builders
    (``take`` / ``__getitem__`` / ``in``), undoing the q/k row permutation of
    ``llama``-architecture files. With a CUDA ``device`` every quantised tensor
    is expanded on the GPU."""

    def __init__(self, path: str, device=None, dtype: torch.dtype = torch.bfloat16):
        self.reader = GGUFReader(path)
        self.config = config_from_metadata(self.reader.metadata, self.reader.tensors)
        self.arch = self.reader.metadata.get("general.architecture", "llama")
        self.device, self.dtype = device, dtype
        self._names = {}
        for n in self.reader.keys():
            h = gguf_to_hf_name(n)
            if h is not None:
                self._names[h] = n

    def keys(self):
        return list(self._names)

    def __contains__(self, name: str) -> bool:
        return name in self._names

    def __getitem__(self, name: str) -> torch.Tensor:
        return self.take(name)

    def take(self, name: str) -> torch.Tensor:
        t = self.reader.get(self._names[name], self.dtype, self.device)
        if self.arch in ("llama", "mistral"):
            c = self.config
            if name.endswith("self_attn.q_proj.weight"):
                t = unpermute_qk(t, c.num_attention_heads)
            elif name.endswith("self_attn.k_proj.weight"):
                t = unpermute_qk(t, c.num_key_value_heads)
        return t

    def items(self):
        for n in self._names:
            yield n, self.take(n)


def save_gguf(path: str, tensors: dict[str, torch.Tensor], cfg, kind: str = "Q8_0", arch: str | None = None,
              keep_f32=("norm",)):
    """Write HF-named tensors as a GGUF file (llama-family names, q/k rows
    permuted for ``llama`` / ``mistral``); 1-D and norm tensors stay F32."""
    arch = arch or {"llama": "llama", "mistral": "mistral", "qwen2": "qwen2"}.get(cfg.model_type, "qwen3")
    w = GGUFWriter(path)
    w.add("general.architecture", arch)
    for key, val in (("block_count", cfg.num_hidden_layers), ("embedding_length", cfg.hidden_size),
                     ("feed_forward_length", cfg.intermediate_size), ("attention.head_count", cfg.num_attention_heads),
                     ("attention.head_count_kv", cfg.num_key_value_heads), ("attention.key_length", cfg.head_dim),
                     ("context_length", cfg.max_position_embeddings)):
        w.add(f"{arch}.{key}", int(val))
    w.add(f"{arch}.attention.layer_norm_rms_epsilon", float(cfg.rms_norm_eps))
    w.add(f"{arch}.rope.freq_base", float(cfg.rope_theta))
    for name, t in tensors.items():
        g = hf_to_gguf_name(name)
        if g is None:
            continue
        t = t.float()
        if arch in ("llama", "mistral"):
            if name.endswith("self_attn.q_proj.weight"):
                t = permute_qk(t, cfg.num_attention_heads)
            elif name.endswith("self_attn.k_proj.weight"):
                t = permute_qk(t, cfg.num_key_value_heads)
        be = GGML_TYPES[TYPE_ID[kind]][1]
        k = "F32" if (t.dim() == 1 or any(s in name for s in keep_f32) or t.shape[-1] % be) else kind
        w.add_tensor(g, t, k)
    w.write()
    return path
