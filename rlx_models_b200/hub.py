"""Model hub: ``org/repo[:QUANT][@rev]`` references resolved to a local
directory (offline first).

* ``select_files(files, quant)``: the files a model needs from a repository
  listing - one GGUF file (the requested quant, else the preference order
  Q4_K_M, Q4_K_S, Q5_K_M, Q6_K, Q8_0, ...) when the repository ships GGUF,
  otherwise config / tokenizer / safetensors files (plus the index);
* ``resolve(ref)``: a local path, or the snapshot in the HF cache, or - with
  ``download=True`` and network access - a download of only the selected
  files through ``huggingface_hub`` into that cache.

Reference: crates/rlx-model-hub (model_ref.rs: ref syntax; quant.rs: quant
preference; resolve.rs: cache + download).
"""
from __future__ import annotations

import fnmatch
import os

from .api import GGUF_QUANT_PREFERENCE, parse_model_ref, resolve_model_path

ESSENTIAL = ("config.json", "generation_config.json", "tokenizer.json", "tokenizer_config.json",
             "tokenizer.model", "vocab.json", "merges.txt", "special_tokens_map.json", "chat_template.jinja",
             "*.safetensors", "*.safetensors.index.json", "preprocessor_config.json")


def select_files(files: list[str], quant: str | None = None) -> list[str]:
    ggufs = sorted(f for f in files if f.lower().endswith(".gguf"))
    if ggufs:
        for q in ((quant,) if quant else GGUF_QUANT_PREFERENCE):  # a requested quant must exist
            hit = [f for f in ggufs if q.lower() in os.path.basename(f).lower()]
            if hit:
                # split GGUF files (-00001-of-0000N) travel together
                base = hit[0].split("-00001-of-")[0]
                return sorted(f for f in ggufs if f.startswith(base)) if "-00001-of-" in hit[0] else [hit[0]]
        if quant:
            raise FileNotFoundError(f"no GGUF file for quant {quant!r}: {ggufs}")
        return [ggufs[0]]
    return sorted(f for f in files if any(fnmatch.fnmatch(os.path.basename(f), p) for p in ESSENTIAL))


def resolve(ref: str, *, download: bool = False, cache_dir: str | None = None, api=None) -> str:
    """Local directory (or .gguf file) for ``ref``; ``api`` is a stand-in for
    ``huggingface_hub`` in tests (list_repo_files / snapshot_download)."""
    p = resolve_model_path(ref)
    name, quant, rev = parse_model_ref(ref)
    if p is not None and not (quant and os.path.isdir(p) and not any(quant.lower() in f.lower()
                                                                     for f in os.listdir(p))):
        return p
    if not download:
        raise FileNotFoundError(f"{ref!r} is not local or in the HF cache (pass download=True to fetch it)")
    if api is None:
        import huggingface_hub as api  # noqa: N813
    files = api.list_repo_files(name, revision=rev)
    want = select_files(files, quant)
    return api.snapshot_download(name, revision=rev, allow_patterns=want, cache_dir=cache_dir)
