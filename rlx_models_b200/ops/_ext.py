"""Loader for the in-tree sm_100a extension and per-device scratch buffers.

The kernels live in ``rlx_models_b200/_C*.so`` (built by ``setup.py
build_ext --inplace``). There is no silent fallback: if a CUDA device is
present and the extension is missing, the first op call raises.
"""
from __future__ import annotations

import threading

import torch

_C = None
_ERR = None
try:  # the .so imports fine on machines without a GPU
    from rlx_models_b200 import _C as _C  # type: ignore
except Exception as e:  # pragma: no cover - only when not built
    _ERR = e


def ext():
    if _C is None:
        raise RuntimeError(
            "rlx_models_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {_ERR})")
    return _C


def available() -> bool:
    return _C is not None and torch.cuda.is_available()


class DeviceScratch:
    """Scratch memory shared by all kernel launches on one device/stream order.

    * ``status``: int32[4] device error word written by bounded waits.
    * ``gemm_ws`` / ``gemm_sem``: split-K partial tiles and per-tile semaphores
      (semaphores are self-resetting, so they start and stay zero).
    * ``attn_ws``: split-KV partial outputs of decode attention.
    """

    GEMM_WS_ELEMS = 12 * 1024 * 1024  # fp32, 48 MB
    GEMM_SEM_ELEMS = 65536
    ATTN_WS_ELEMS = 8 * 1024 * 1024  # fp32, 32 MB
    ACC_ELEMS = 128 * 32768  # fp32, 16 MB: [tokens <= 128, features <= 32768]

    def __init__(self, device: torch.device):
        self.device = device
        self.status = torch.zeros(4, dtype=torch.int32, device=device)
        # split-K fp32 tile accumulators: zero at rest (each tile's last split re-zeroes it)
        self.gemm_ws = torch.zeros(self.GEMM_WS_ELEMS, dtype=torch.float32, device=device)
        self.gemm_sem = torch.zeros(self.GEMM_SEM_ELEMS, dtype=torch.int32, device=device)
        self.attn_ws = torch.empty(self.ATTN_WS_ELEMS, dtype=torch.float32, device=device)
        # fp32 sums of the accumulate-only (decode) GEMMs: zero at rest, every
        # consumer kernel zeroes what it reads; one GEMM uses it at a time
        self.acc = torch.zeros(self.ACC_ELEMS, dtype=torch.float32, device=device)

    def acc_view(self, m: int, n: int) -> torch.Tensor:
        assert m * n <= self.ACC_ELEMS, "decode accumulator too small"
        return self.acc[:m * n].view(m, n)

    def check(self):
        """Raise if any kernel on this device recorded an error (syncs)."""
        st = self.status.cpu().tolist()
        if st[0] != 0:
            self.status.zero_()
            raise KernelError(st)


class KernelError(RuntimeError):
    CODES = {
        1: "TMA stage wait timed out", 2: "free-stage wait timed out",
        3: "accumulator wait timed out", 4: "accumulator release wait timed out",
        5: "peer flag wait timed out", 6: "split-K wait timed out", 7: "bounds check failed",
        8: "drain wait timed out", 9: "test timeout",
    }

    def __init__(self, st):
        self.code, self.block, self.thread, self.detail = st
        super().__init__(
            f"b200 kernel error {self.code} ({self.CODES.get(self.code, '?')}) "
            f"block={self.block} thread={self.thread} detail={self.detail}")


_LAUNCHES = [0]


def count_launches(n: int = 1) -> None:
    """Host-side tally of this package's kernel launches (eager calls and
    graph captures); graph replays are added by the engine."""
    _LAUNCHES[0] += int(n)


def launch_count() -> int:
    return _LAUNCHES[0]


_scratch: dict[tuple[int, int], DeviceScratch] = {}
_lock = threading.Lock()
_slot = threading.local()


class scratch_slot:
    """Context manager: kernels launched inside use scratch set ``i`` of the
    device. Work queued on two streams at once (e.g. two prefill micro-batches
    overlapping one's collective with the other's GEMMs) must use different
    slots, since split-K workspaces and semaphores are per set."""

    def __init__(self, i: int):
        self.i = int(i)

    def __enter__(self):
        self.prev = getattr(_slot, "i", 0)
        _slot.i = self.i
        return self

    def __exit__(self, *exc):
        _slot.i = self.prev
        return False


def scratch(device: torch.device | int | None = None) -> DeviceScratch:
    if device is None:
        device = torch.cuda.current_device()
    idx = device.index if isinstance(device, torch.device) else int(device)
    if idx is None:
        idx = torch.cuda.current_device()
    key = (idx, getattr(_slot, "i", 0))
    s = _scratch.get(key)
    if s is None:
        with _lock:
            s = _scratch.get(key)
            if s is None:
                s = DeviceScratch(torch.device("cuda", idx))
                _scratch[key] = s
    return s


def check_errors(device=None):
    if device is None:
        device = torch.cuda.current_device()
    idx = device.index if isinstance(device, torch.device) else int(device)
    if idx is None:
        idx = torch.cuda.current_device()
    for (d, _), s in list(_scratch.items()):
        if d == idx:
            s.check()
    if (idx, 0) not in _scratch:
        scratch(device).check()
