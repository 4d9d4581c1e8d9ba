"""Model plugins: open any checkpoint through a registry of providers and use
it through one task-level interface.

A provider answers ``can_open(path, options)`` and ``open(path, options)``;
``open_model`` asks the registered providers in order (most recent first).
The built-in ``rlx_models_b200`` provider opens whatever ``api.load``
resolves - a safetensors directory, a ``.gguf`` file or a directory of them,
an MLX-quantised directory, an HF id in the offline cache, or a named shape -
and returns a :class:`PluginModel` with ``info``, ``generate_text``,
``chat``, ``embed`` and ``logits``. Text generation stops at the usual
end-of-turn tokens of the supported families. A task beyond text (speech,
vision) is one more provider registered the same way.

Open options: ``device`` (default "cuda"), ``max_seq`` (context in tokens),
``tokenizer`` (a tokenizer directory; default next to the weights),
``tp_rank`` / ``tp_size`` / ``comm`` for tensor-parallel ranks.

Reference: crates/rlx-models-plugin/src/lib.rs (`RlxModelsProvider`, open
options device / max_seq / tokenizer, end-of-turn stop tokens), tasks.rs.
"""
from __future__ import annotations

import os
from typing import Protocol

STOP_TOKENS = ("<|endoftext|>", "<|im_end|>", "<|eot_id|>", "<|end|>", "<end_of_turn>", "</s>", "<|return|>")
KNOWN_OPTIONS = {"device", "max_seq", "tokenizer", "tp_rank", "tp_size", "comm", "seed"}


class ModelProvider(Protocol):
    name: str

    def can_open(self, path: str, options: dict) -> bool: ...

    def open(self, path: str, options: dict): ...


class PluginModel:
    """Task-level facade over a loaded :class:`~rlx_models_b200.api.LLM`."""

    def __init__(self, llm, source: str, provider: str):
        self.llm, self.source, self.provider = llm, source, provider
        tok = llm.tokenizer
        self.stop_ids = []
        if tok is not None and hasattr(tok, "encode"):
            for s in STOP_TOKENS:
                try:
                    ids = tok.encode(s)
                except Exception:
                    continue
                if len(ids) == 1:
                    self.stop_ids.append(ids[0])
            eos = getattr(tok, "eos_token_id", None)
            if eos is not None and eos not in self.stop_ids:
                self.stop_ids.append(int(eos))

    def info(self) -> dict:
        c = self.llm.config
        return {"provider": self.provider, "source": self.source, "model_type": c.model_type,
                "layers": c.num_hidden_layers, "hidden": c.hidden_size, "vocab": c.vocab_size,
                "tasks": ["text-generation", "chat", "embeddings", "logits"]}

    def _params(self, max_tokens, sampling):
        from .runtime.engine import SamplingParams
        return SamplingParams(max_new_tokens=int(max_tokens), stop_token_ids=list(self.stop_ids), **sampling)

    def _decode(self, toks):
        tok = self.llm.tokenizer
        toks = [t for t in toks if t not in self.stop_ids]
        return tok.decode(toks) if tok is not None else toks

    def generate_text(self, prompt, max_tokens: int = 64, **sampling):
        out = self.llm.generate(prompt, self._params(max_tokens, sampling))[0]
        return self._decode(out.token_ids)

    def chat(self, messages: list[dict], max_tokens: int = 128, tools=None, **sampling):
        tok = self.llm.tokenizer
        if tok is None:
            raise ValueError("chat needs a tokenizer")
        try:
            text = tok.apply_chat_template(messages, add_generation_prompt=True, tokenize=False, tools=tools)
        except TypeError:
            text = tok.apply_chat_template(messages, add_generation_prompt=True, tokenize=False)
        return self.generate_text(text, max_tokens, **sampling)

    def embed(self, texts, pooling: str = "last", normalize: bool = True):
        return self.llm.embed(texts, pooling=pooling, normalize=normalize)

    def logits(self, prompt):
        return self.llm.logits(prompt)


class RlxModelsProvider:
    name = "rlx_models_b200"

    def can_open(self, path: str, options: dict) -> bool:
        from .api import resolve_model_path
        from .config import PRESETS
        if path in PRESETS:
            return True
        p = resolve_model_path(path)
        if p is None:
            return False
        if os.path.isfile(p):
            return p.lower().endswith(".gguf")
        return os.path.exists(os.path.join(p, "config.json")) or any(
            f.lower().endswith(".gguf") for f in os.listdir(p))

    def open(self, path: str, options: dict) -> PluginModel:
        from .api import load
        from .runtime.engine import EngineConfig
        ecfg = EngineConfig(max_model_len=int(options.get("max_seq", 4096)))
        llm = load(path, device=options.get("device", "cuda"), tp_rank=int(options.get("tp_rank", 0)),
                   tp_size=int(options.get("tp_size", 1)), comm=options.get("comm"), seed=int(options.get("seed", 0)),
                   engine_config=ecfg)
        if options.get("tokenizer"):
            from .tokenizer import load_tokenizer
            llm.tokenizer = load_tokenizer(options["tokenizer"])
        return PluginModel(llm, path, self.name)


_PROVIDERS: list = [RlxModelsProvider()]


def register_provider(provider) -> None:
    """Add a provider; it is asked before the ones registered earlier."""
    _PROVIDERS.insert(0, provider)


def providers() -> list[str]:
    return [p.name for p in _PROVIDERS]


def open_model(path: str, options: dict | None = None):
    options = dict(options or {})
    unknown = set(options) - KNOWN_OPTIONS - set(options.get("_extra_keys", ()))
    if unknown:
        raise ValueError(f"unknown open options {sorted(unknown)}; known: {sorted(KNOWN_OPTIONS)}")
    for p in _PROVIDERS:
        if p.can_open(path, options):
            return p.open(path, options)
    raise FileNotFoundError(f"no model provider can open {path!r} (providers: {providers()})")
