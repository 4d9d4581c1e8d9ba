"""Configuration: one registry of environment knobs, and typed run configs
loadable from a YAML / JSON file.

Knobs. Every environment switch the package reads is declared once in
``KNOBS`` (name, type, default, who reads it, what it does). ``get(name)``
resolves a value with the precedence code override > process environment >
default; ``override(name, value)`` sets a code override and also exports it to
``os.environ``, because the CUDA side reads its switches with ``getenv`` the
first time the kernel family launches (so overrides of CUDA knobs must be set
before the first launch). ``describe()`` renders the table that ``serve`` /
``run`` / ``train`` print at startup with ``--show-knobs`` and that
``python -m rlx_models_b200 knobs`` prints.

Run configs. ``RunConfig`` groups the typed sections a run needs:

    model: qwen3-8b                  # id, preset or path
    parallel: {tp: 8, tp_comm: pull} # ParallelConfig
    serve: {max_num_seqs: 64, kv_memory_gb: 40}   # runtime.engine.EngineConfig fields
    train: {lr: 1.0e-4, optimizer: muon}          # train.trainer.TrainConfig fields
    kernel: {B200_PDL: 1}            # knob overrides

``load_run_config(path)`` reads such a file; unknown keys are errors that list
the valid ones. The CLI's ``--config FILE`` fills the engine / trainer
settings from it; explicit command-line flags still win.

Reference: the reference reads its ``RLX_*`` settings only through one
accessor where a code override wins over the process environment
(README.md:641-653) and keeps per-model compile profiles in ``*.rlx.toml``
files (crates/rlx-models-core/src/flow_bridge.rs:118-230).
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any


@dataclass(frozen=True)
class Knob:
    name: str
    kind: str          # "bool" | "int" | "str"
    default: Any
    reader: str        # "python" | "cuda" | "build"
    help: str
    choices: tuple = ()


KNOBS: dict[str, Knob] = {k.name: k for k in [
    Knob("B200_PDL", "bool", True, "cuda",
         "programmatic dependent launch on every kernel launch (0: plain launches, e.g. for per-kernel timing)"),
    Knob("B200_ATTN_LEGACY", "bool", False, "cuda",
         "force the mma.sync prefill attention instead of the tcgen05 FMHA"),
    Knob("B200_DECODE_CHUNK", "int", 0, "cuda",
         "decode attention: fixed KV pages per CTA instead of equal splits (0: off; measured slower)"),
    Knob("B200_MOE_DEBUG", "int", 0, "cuda", "MoE grouped GEMM timing experiments (bit flags; 0 in production)"),
    Knob("B200_GEMM_TRACE", "bool", False, "build",
         "compile the per-CTA GEMM timeline probes (setup.py; read by bench/gemm_trace.py)"),
    Knob("B200_DEBUG_CHECKS", "bool", False, "build", "compile device bounds checks into the kernels (setup.py)"),
    Knob("B200_PTXAS_VERBOSE", "bool", False, "build", "print ptxas register / spill reports while building"),
    Knob("B200_TP_TWO_SHOT", "str", "auto", "python",
         "tensor-parallel decode reduction: auto (two-shot from 8 ranks and 16 rows), on, off", ("auto", "on", "off")),
    Knob("B200_TP_PREFILL_OVERLAP", "bool", True, "python",
         "split long TP prefill steps into two micro-batches whose all-reduces overlap"),
    Knob("B200_NVTX", "bool", False, "python", "NVTX ranges per layer / engine step / training phase"),
    Knob("RLX_B200_ASSET_CACHE", "str", "~/.cache/rlx_models_b200/assets", "python",
         "where .rlxp asset packs are materialised"),
    Knob("RLX_WEIGHTS_DIR", "str", "", "python", "first root searched by weight discovery"),
    Knob("RLX_WEIGHTS_PATHS", "str", "", "python", "extra discovery roots (os.pathsep-separated)"),
]}

_OVERRIDES: dict[str, Any] = {}


def _parse(k: Knob, raw: Any) -> Any:
    if k.kind == "bool":
        if isinstance(raw, bool):
            return raw
        return str(raw).strip().lower() not in ("0", "false", "no", "off", "")
    if k.kind == "int":
        return int(raw)
    v = str(raw)
    if k.choices and v not in k.choices:
        raise ValueError(f"{k.name}={v!r}: expected one of {k.choices}")
    return v


def _env_str(k: Knob, v: Any) -> str:
    if k.kind == "bool":
        return "1" if v else "0"
    return str(v)


def get(name: str) -> Any:
    """Value of a declared knob: code override > environment > default."""
    k = KNOBS[name]
    if name in _OVERRIDES:
        return _OVERRIDES[name]
    raw = os.environ.get(name)
    return k.default if raw is None else _parse(k, raw)


def source(name: str) -> str:
    return "override" if name in _OVERRIDES else ("env" if name in os.environ else "default")


def override(name: str, value: Any) -> None:
    """Set a knob from code (wins over the environment). CUDA-side knobs take
    effect for kernel families that have not launched yet in this process."""
    if name not in KNOBS:
        raise KeyError(f"unknown knob {name!r}; known: {sorted(KNOBS)}")
    k = KNOBS[name]
    v = _parse(k, value)
    _OVERRIDES[name] = v
    os.environ[name] = _env_str(k, v)


def clear_overrides() -> None:
    for name in list(_OVERRIDES):
        _OVERRIDES.pop(name)


def describe() -> str:
    rows = [("knob", "value", "source", "read by", "meaning")]
    for name, k in KNOBS.items():
        rows.append((name, str(get(name)), source(name), k.reader, k.help))
    w = [max(len(r[i]) for r in rows) for i in range(4)]
    return "\n".join(f"{r[0]:<{w[0]}}  {r[1]:<{w[1]}}  {r[2]:<{w[2]}}  {r[3]:<{w[3]}}  {r[4]}" for r in rows)


# ---------------------------------------------------------------------------
# typed run configs
# ---------------------------------------------------------------------------

@dataclass
class ParallelConfig:
    tp: int = 1
    ep: int = 1
    pp: int = 1
    fsdp: int = 1
    sp: int = 1
    tp_comm: str = "pull"   # nccl | fused | pull

    def world(self) -> int:
        return self.tp * self.ep * self.pp * self.fsdp * self.sp


@dataclass
class RunConfig:
    model: str | None = None
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    serve: dict = field(default_factory=dict)   # EngineConfig fields
    train: dict = field(default_factory=dict)   # TrainConfig fields
    kernel: dict = field(default_factory=dict)  # knob overrides

    def engine_config(self, **cli):
        """EngineConfig from the ``serve`` section; keyword arguments (explicit
        command-line values) win."""
        from .runtime.engine import EngineConfig
        return EngineConfig(**{**self.serve, **cli})

    def train_config(self, **cli):
        from .train.trainer import TrainConfig
        return TrainConfig(**{**self.train, **cli})

    def apply_kernel_overrides(self) -> None:
        for name, v in self.kernel.items():
            override(name, v)


def _check_keys(section: str, d: dict, cls) -> None:
    names = {f.name for f in dataclasses.fields(cls)}
    bad = sorted(set(d) - names)
    if bad:
        raise ValueError(f"config section {section!r}: unknown keys {bad}; valid: {sorted(names)}")


def run_config_from_dict(d: dict) -> RunConfig:
    from .runtime.engine import EngineConfig
    from .train.trainer import TrainConfig
    _check_keys("top level", d, RunConfig)
    par = dict(d.get("parallel") or {})
    _check_keys("parallel", par, ParallelConfig)
    serve = dict(d.get("serve") or {})
    _check_keys("serve", serve, EngineConfig)
    train = dict(d.get("train") or {})
    _check_keys("train", train, TrainConfig)
    for k in ("betas", "lora_targets", "graph_batch_sizes", "kv_cache_scales"):
        for sec in (serve, train):
            if k in sec and isinstance(sec[k], list):
                sec[k] = tuple(sec[k])
    kernel = dict(d.get("kernel") or {})
    unknown = sorted(set(kernel) - set(KNOBS))
    if unknown:
        raise ValueError(f"config section 'kernel': unknown knobs {unknown}; known: {sorted(KNOBS)}")
    for name, v in kernel.items():
        _parse(KNOBS[name], v)
    return RunConfig(model=d.get("model"), parallel=ParallelConfig(**par), serve=serve, train=train, kernel=kernel)


def load_run_config(path: str) -> RunConfig:
    """RunConfig from a .yaml / .yml / .json file."""
    with open(path) as f:
        text = f.read()
    if path.endswith((".yaml", ".yml")):
        import yaml
        d = yaml.safe_load(text) or {}
    else:
        d = json.loads(text)
    if not isinstance(d, dict):
        raise ValueError(f"{path}: expected a mapping at the top level")
    return run_config_from_dict(d)
