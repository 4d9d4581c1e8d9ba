"""Tool calls in generated text.

Qwen / Hermes-style chat templates make the model emit each call as a JSON
object ``{"name": ..., "arguments": {...}}`` wrapped in
``<tool_call> ... </tool_call>``; some models emit the bare object. ``parse``
returns the calls and the remaining text; ``to_openai`` validates each call
against the request's tools (serve/guardrails.py), sanitises its arguments and
produces the OpenAI ``tool_calls`` entries, collecting rejected calls
separately.

Reference: crates/rlx-qwen3/src/tool_call.rs (parsing), rlx-guardrails
(validation) on the rlx-serve chat route.
"""
from __future__ import annotations

import json
import re
import uuid

from . import guardrails as GR

_BLOCK = re.compile(r"<tool_call>\s*(.*?)\s*(?:</tool_call>|$)", re.S)


def _as_call(obj) -> dict | None:
    if isinstance(obj, dict) and isinstance(obj.get("name"), str):
        args = obj.get("arguments", obj.get("parameters", {}))
        return {"name": obj["name"], "arguments": args}
    return None


def parse(text: str) -> tuple[list[dict], str]:
    """-> (calls [{"name", "arguments"}], text outside the call blocks)."""
    calls = []
    if "<tool_call>" in text:
        for m in _BLOCK.finditer(text):
            try:
                c = _as_call(json.loads(m.group(1)))
            except ValueError:
                c = None
            if c is not None:
                calls.append(c)
        rest = _BLOCK.sub("", text).strip()
        return calls, rest
    s = text.strip()
    if s.startswith("{") and s.endswith("}"):
        try:
            c = _as_call(json.loads(s))
        except ValueError:
            c = None
        if c is not None:
            return [c], ""
    return [], text


def to_openai(calls: list[dict], tools: list[dict]) -> tuple[list[dict], list[str]]:
    out, errors = [], []
    for c in calls:
        try:
            GR.validate_tool_call(c, tools)
            args = GR.sanitize_tool_arguments(c, tools)
        except GR.GuardrailError as e:
            errors.append(str(e))
            continue
        out.append({"id": "call_" + uuid.uuid4().hex[:24], "type": "function",
                    "function": {"name": c["name"], "arguments": GR.arguments_wire_string(args)}})
    return out, errors
