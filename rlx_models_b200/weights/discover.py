"""Find model weights that other local tools already downloaded (no network).

``scan`` walks the caches of common LLM apps and lists loadable weights;
``resolve`` turns a short query ("qwen3-0.6b", "ollama:qwen2.5:32b") into a
path that :func:`rlx_models_b200.api.load` accepts.

| source       | roots (environment override first)                                          |
|--------------|-----------------------------------------------------------------------------|
| local        | ``RLX_WEIGHTS_DIR``, ``./weights``                                          |
| LM Studio    | ``LMS_MODELS`` / ``LM_STUDIO_MODELS``, ``~/.lmstudio/models``               |
| Ollama       | ``OLLAMA_MODELS``, ``~/.ollama/models``, ``/usr/share/ollama/.ollama/models`` |
| Hugging Face | ``HF_HUB_CACHE``, ``$HF_HOME/hub``, ``~/.cache/huggingface/hub``            |
| extra        | ``RLX_WEIGHTS_PATHS`` (``os.pathsep``-separated)                            |

Recognised: GGUF files (by their magic), safetensors model directories
(``config.json`` next to ``*.safetensors``), and Ollama manifests whose model
layer is a GGUF blob (``manifests/<registry>/<ns>/<name>/<tag>`` ->
``blobs/sha256-<digest>``, shown as ``ollama:<name>:<tag>``).

Reference: rlx-models-core src/weights_discover.rs (``scan_weights``,
``resolve_weight_query``, Ollama manifests :992-1060).
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass

SOURCES = ("local", "lmstudio", "ollama", "hf", "extra")
_PRIORITY = {k: i for i, k in enumerate(SOURCES)}  # earlier wins when a query matches several


@dataclass
class Hit:
    path: str      # file (GGUF) or directory (safetensors checkpoint)
    source: str    # one of SOURCES
    name: str      # display name used for matching
    fmt: str       # "gguf" | "safetensors"


def _env_paths(*keys: str) -> list[str]:
    out = []
    for k in keys:
        v = os.environ.get(k)
        if v:
            out += [p for p in v.split(os.pathsep) if p]
    return out


def default_roots() -> list[tuple[str, str]]:
    home = os.path.expanduser("~")
    roots = [("local", p) for p in _env_paths("RLX_WEIGHTS_DIR") + [os.path.join(os.getcwd(), "weights")]]
    roots += [("lmstudio", p) for p in (_env_paths("LMS_MODELS", "LM_STUDIO_MODELS")
                                        or [os.path.join(home, ".lmstudio", "models")])]
    roots += [("ollama", p) for p in (_env_paths("OLLAMA_MODELS")
                                      or [os.path.join(home, ".ollama", "models"), "/usr/share/ollama/.ollama/models"])]
    hf = _env_paths("HF_HUB_CACHE") or [os.path.join(os.environ.get("HF_HOME", os.path.join(home, ".cache",
                                                                                              "huggingface")), "hub")]
    roots += [("hf", p) for p in hf]
    roots += [("extra", p) for p in _env_paths("RLX_WEIGHTS_PATHS")]
    return roots


def is_gguf(path: str) -> bool:
    try:
        with open(path, "rb") as f:
            return f.read(4) == b"GGUF"
    except OSError:
        return False


def _hf_name(root: str, path: str) -> str:
    rel = os.path.relpath(path, root).replace(os.sep, "/")
    head = rel.split("/", 1)[0]
    if head.startswith("models--"):  # models--org--repo/snapshots/<rev>/...
        repo = head[len("models--"):].replace("--", "/")
        tail = rel.split("/", 3)[3] if rel.count("/") >= 3 else ""
        return repo + ("/" + tail if tail else "")
    return rel


def _scan_ollama(root: str, hits: list[Hit]):
    manifests, blobs = os.path.join(root, "manifests"), os.path.join(root, "blobs")
    if not (os.path.isdir(manifests) and os.path.isdir(blobs)):
        return
    for dirpath, _, files in os.walk(manifests):
        for fn in files:
            mpath = os.path.join(dirpath, fn)
            try:
                layers = json.load(open(mpath)).get("layers", [])
            except (OSError, ValueError):
                continue
            layer = next((l for l in layers if l.get("mediaType") == "application/vnd.ollama.image.model"), None)
            if layer is None:
                continue
            blob = os.path.join(blobs, layer.get("digest", "").replace(":", "-"))
            if not os.path.isfile(blob) or not is_gguf(blob):
                continue  # non-GGUF model layers are not loadable here
            parts = os.path.relpath(mpath, manifests).replace(os.sep, "/").split("/")
            name, tag = (parts[-2], parts[-1]) if len(parts) >= 2 else (parts[-1], "latest")
            hits.append(Hit(blob, "ollama", f"ollama:{name}:{tag}", "gguf"))


def scan(roots: list[tuple[str, str]] | None = None, query: str | None = None, max_depth: int = 8) -> list[Hit]:
    """Every loadable checkpoint under ``roots`` (default: ``default_roots()``),
    optionally filtered by a case-insensitive substring of its name."""
    hits: list[Hit] = []
    for source, root in (roots if roots is not None else default_roots()):
        if not os.path.isdir(root):
            continue
        if source == "ollama":
            _scan_ollama(root, hits)
            continue
        base_depth = root.rstrip(os.sep).count(os.sep)
        for dirpath, dirs, files in os.walk(root):
            if dirpath.count(os.sep) - base_depth >= max_depth:
                dirs[:] = []
            dirs[:] = [d for d in dirs if not d.startswith(".") and d != "blobs"]
            name_of = (lambda p: _hf_name(root, p)) if source == "hf" else \
                (lambda p: os.path.relpath(p, root).replace(os.sep, "/"))
            if "config.json" in files and any(f.endswith(".safetensors") for f in files):
                hits.append(Hit(dirpath, source, name_of(dirpath), "safetensors"))
            for fn in files:
                if fn.lower().endswith(".gguf"):
                    p = os.path.join(dirpath, fn)
                    if is_gguf(p):
                        hits.append(Hit(p, source, name_of(p), "gguf"))
    if query:
        q = query.lower()
        hits = [h for h in hits if q in h.name.lower() or q in os.path.basename(h.path).lower()]
    return hits


def resolve(query: str, roots: list[tuple[str, str]] | None = None, prefer_quant: str = "Q4_K_M") -> str | None:
    """Best local path for ``query``: an exact display-name match first, then
    names containing the query; among GGUF files the preferred quantisation,
    then source priority (local, LM Studio, Ollama, HF cache, extra)."""
    hits = scan(roots, query)
    if not hits:
        return None
    q = query.lower()

    def key(h: Hit):
        exact = h.name.lower() == q or h.name.lower().rstrip("/").endswith("/" + q)
        quant = prefer_quant.lower() in os.path.basename(h.path).lower() if h.fmt == "gguf" else True
        return (not exact, not quant, _PRIORITY.get(h.source, 99), len(h.name))

    return min(hits, key=key).path
