"""Tokenizers: the checkpoint's own (HF ``tokenizer.json`` / ``tokenizer_config.json``
through transformers, offline) or, for random-weight shapes, a byte-level
fallback (UTF-8 bytes -> ids 0..255, so text prompts work end to end).

Reference: the runners load ``tokenizer.json`` next to the weights
(rlx-qwen3 src/high_level_runner.rs, rlx-models-core src/tokenizer*.rs).
"""
from __future__ import annotations

import json
import os


class ByteTokenizer:
    """UTF-8 bytes as token ids (ids >= 256 decode to nothing)."""
    eos_token_id = None
    chat_template = None

    def encode(self, text: str) -> list[int]:
        return list(text.encode("utf-8"))

    def decode(self, ids) -> str:
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=False, tools=None):
        s = ""
        if tools:  # tool catalog as a system block; calls come back as <tool_call>{json}</tool_call>
            s += "<|system|>\n# Tools\n" + "\n".join(json.dumps(t) for t in tools) + \
                 "\nCall a tool with <tool_call>{\"name\": ..., \"arguments\": {...}}</tool_call>\n"
        s += "".join(f"<|{m['role']}|>\n{m.get('content') or ''}\n" for m in messages)
        return s + ("<|assistant|>\n" if add_generation_prompt else "")


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer
        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.eos_token_id = self.tok.eos_token_id
        self.chat_template = getattr(self.tok, "chat_template", None)

    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text, add_special_tokens=False)

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids), skip_special_tokens=True)

    def apply_chat_template(self, messages, add_generation_prompt=True, tokenize=False, tools=None):
        if self.chat_template:
            return self.tok.apply_chat_template(messages, add_generation_prompt=add_generation_prompt,
                                                tokenize=tokenize, tools=tools)
        return ByteTokenizer().apply_chat_template(messages, add_generation_prompt, tools=tools)


def load_tokenizer(path: str | None):
    if path and any(os.path.exists(os.path.join(path, f)) for f in ("tokenizer.json", "tokenizer_config.json",
                                                                       "tokenizer.model")):
        return HFTokenizer(path)
    return ByteTokenizer()
