"""Tracing and inspection.

* Tensor inspection: ``enable_inspect()`` makes the models record, per named
  tensor (each layer's output, the final hidden states), the count of NaN /
  Inf values, min, max, mean, absolute max and a 16-bin histogram;
  ``take_inspect_log()`` returns and clears the records. Recording happens
  only in eager execution (never while a CUDA graph is being captured) and
  costs nothing when disabled.
* NVTX ranges: with ``B200_NVTX=1`` (or ``enable_nvtx()``) every decoder
  layer, engine step and training phase is wrapped in an NVTX range, so an
  Nsight Systems timeline (or any NVTX consumer) shows the model structure.
* ``profile(fn, ...)``: run ``fn`` under the torch profiler (CUPTI device
  activity), write a Chrome trace and return the top kernels by device time;
  ``python -m rlx_models_b200 profile`` drives it over engine steps.

Reference: the reference's `enable_inspect` / `take_inspect_log`
(crates/rlx-qwen3/src/high_level_runner.rs:857-870) and its CUDA step
profiler (`RLX_CUDA_STEP_PROFILE`, crates/rlx-ling/README.md:445-462).
"""
from __future__ import annotations

import contextlib
import os

import torch

_INSPECT = {"on": False, "log": []}
_NVTX = {"on": os.environ.get("B200_NVTX", "0") == "1"}


def enable_inspect(on: bool = True):
    _INSPECT["on"] = on


def inspecting() -> bool:
    return _INSPECT["on"]


def take_inspect_log() -> list[dict]:
    log, _INSPECT["log"] = _INSPECT["log"], []
    return log


def inspect(name: str, t: torch.Tensor):
    if not _INSPECT["on"]:
        return
    if t.is_cuda and torch.cuda.is_current_stream_capturing():
        return
    x = t.detach().float()
    finite = torch.isfinite(x)
    xf = x[finite]
    rec = {"name": name, "shape": tuple(t.shape), "dtype": str(t.dtype).replace("torch.", ""),
           "nan": int(torch.isnan(x).sum()), "inf": int(torch.isinf(x).sum())}
    if xf.numel():
        lo, hi = float(xf.min()), float(xf.max())
        rec.update(min=lo, max=hi, mean=float(xf.mean()), absmax=max(abs(lo), abs(hi)),
                   hist=torch.histc(xf, bins=16, min=lo, max=hi if hi > lo else lo + 1e-6).int().tolist())
    _INSPECT["log"].append(rec)


def enable_nvtx(on: bool = True):
    _NVTX["on"] = on


@contextlib.contextmanager
def nvtx(name: str):
    if not _NVTX["on"] or not torch.cuda.is_available():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def profile(fn, steps: int = 3, warmup: int = 1, trace_path: str | None = None, top: int = 20) -> list[dict]:
    """Run ``fn()`` ``warmup + steps`` times, profile the last ``steps``;
    returns [{name, calls, device_us_total, device_us_avg}] sorted by device time."""
    from torch.profiler import ProfilerActivity, profile as tprof
    for _ in range(warmup):
        fn()
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    with tprof(activities=acts) as prof:
        for _ in range(steps):
            fn()
        if torch.cuda.is_available():
            torch.cuda.synchronize()
    if trace_path:
        prof.export_chrome_trace(trace_path)
    rows = []
    for e in prof.key_averages():
        dev = getattr(e, "device_time_total", None)
        if dev is None:
            dev = getattr(e, "cuda_time_total", 0.0)
        if dev and dev > 0:
            rows.append({"name": e.key, "calls": int(e.count), "device_us_total": float(dev),
                         "device_us_avg": float(dev) / max(1, int(e.count))})
    rows.sort(key=lambda r: -r["device_us_total"])
    return rows[:top]
