"""Guardrails for the OpenAI-compatible serving path: tool-call validation
and conversation compaction, on plain OpenAI-shaped dicts.

Tool calls: a model's call must name a tool from the request's catalog (names
with the reserved ``_rlx_`` prefix only if the catalog declares them) and
carry every ``required`` argument of the tool's JSON schema. Sanitising keeps
only arguments that the schema declares (or that ``additionalProperties``
admits) and whose value fits the declared ``type`` / ``enum``. Arguments may
arrive as an object or as a JSON string (the wire form); they go back out as a
JSON string that always holds an object.

Compaction: with a token budget, system messages are always kept; the
oldest ``tool`` results go first, then the oldest of any other role, until
the estimate fits. The estimate is the tokenizer's count when one is given,
else about four characters per token.

Reference: crates/rlx-guardrails/src/tools.rs (validate_tool_call :156,
sanitize_tool_arguments :218, tool_arguments_wire_string :240), compact.rs
(compact_messages :77), error.rs.
"""
from __future__ import annotations

import json
from typing import Callable

RESERVED_PREFIX = "_rlx_"
RESPOND_TOOL = "_rlx_respond"
EMIT_STRUCTURED_TOOL = "_rlx_emit_structured"
RESERVED_NAMES = (RESPOND_TOOL, EMIT_STRUCTURED_TOOL)


class GuardrailError(ValueError):
    def __init__(self, kind: str, tool: str, fields: list[str] | None = None):
        self.kind, self.tool, self.fields = kind, tool, list(fields or [])
        msg = {"unknown_tool": f"unknown tool {tool!r}: not in the request's tool set",
               "reserved_tool": f"tool name {tool!r} is reserved for the server",
               "missing_required": f"tool {tool!r} call lacks required arguments {self.fields}"}[kind]
        super().__init__(msg)


def tool_name(tool: dict) -> str:
    return tool.get("function", tool).get("name", "")


def tool_schema(tool: dict) -> dict | None:
    return tool.get("function", tool).get("parameters")


def respond_tool() -> dict:
    """Plain-text reply escape hatch offered next to the caller's tools."""
    return {"type": "function", "function": {"name": RESPOND_TOOL, "parameters": {
        "type": "object", "properties": {"message": {"type": "string"}}, "required": ["message"],
        "additionalProperties": False}}}


def emit_structured_tool(schema: dict) -> dict:
    return {"type": "function", "function": {"name": EMIT_STRUCTURED_TOOL, "parameters": schema}}


def is_reserved(name: str, prefix: str = RESERVED_PREFIX) -> bool:
    return name.startswith(prefix)


def collides_with_reserved(tools: list[dict]) -> bool:
    return any(tool_name(t) in RESERVED_NAMES for t in tools)


def arguments_object(arguments) -> dict | None:
    """object -> itself; JSON string -> the decoded object (None if it is not
    one); None -> None; any other scalar -> {}."""
    if isinstance(arguments, dict):
        return dict(arguments)
    if isinstance(arguments, str):
        try:
            v = json.loads(arguments)
        except ValueError:
            return None
        return v if isinstance(v, dict) else None
    if arguments is None:
        return None
    return {}


def _missing(schema: dict | None, args: dict) -> list[str]:
    if not isinstance(schema, dict):
        return []
    return [f for f in schema.get("required", []) if isinstance(f, str) and f not in args]


def validate_tool_call(call: dict, tools: list[dict]) -> None:
    """``call``: {"name", "arguments"} (or an OpenAI tool_call with "function")."""
    fn = call.get("function", call)
    name = fn.get("name", "")
    declared = {tool_name(t): t for t in tools}
    if is_reserved(name) and name not in declared:
        raise GuardrailError("reserved_tool", name)
    if name not in declared:
        raise GuardrailError("unknown_tool", name)
    args = arguments_object(fn.get("arguments")) or {}
    miss = _missing(tool_schema(declared[name]), args)
    if miss:
        raise GuardrailError("missing_required", name, miss)


_TYPE_CHECKS: dict[str, Callable[[object], bool]] = {
    "array": lambda v: isinstance(v, list),
    "boolean": lambda v: isinstance(v, bool),
    "integer": lambda v: isinstance(v, int) and not isinstance(v, bool),
    "null": lambda v: v is None,
    "number": lambda v: isinstance(v, (int, float)) and not isinstance(v, bool),
    "object": lambda v: isinstance(v, dict),
    "string": lambda v: isinstance(v, str),
}


def _fits(value, schema) -> bool:
    if not isinstance(schema, dict):
        return True
    if isinstance(schema.get("enum"), list) and value not in schema["enum"]:
        return False
    t = schema.get("type")
    if t is None:
        return True
    types = [t] if isinstance(t, str) else [x for x in t if isinstance(x, str)] if isinstance(t, list) else None
    if types is None:
        return True
    return any(_TYPE_CHECKS.get(x, lambda v: True)(value) for x in types)


def sanitize_tool_arguments(call: dict, tools: list[dict]) -> dict:
    """Arguments with undeclared / ill-typed keys removed; raises when a
    required argument does not survive."""
    fn = call.get("function", call)
    args = arguments_object(fn.get("arguments")) or {}
    tool = next((t for t in tools if tool_name(t) == fn.get("name")), None)
    schema = tool_schema(tool) if tool is not None else None
    if not isinstance(schema, dict):
        return args
    props = schema.get("properties")
    if isinstance(props, dict):
        extra = schema.get("additionalProperties")
        allow_extra = extra is True or isinstance(extra, dict)
        args = {k: v for k, v in args.items() if (k in props and _fits(v, props[k])) or (k not in props and allow_extra)}
    miss = _missing(schema, args)
    if miss:
        raise GuardrailError("missing_required", fn.get("name", ""), miss)
    return args


def arguments_wire_string(arguments) -> str:
    """OpenAI wire form: a JSON string holding an object ("{}" otherwise)."""
    if isinstance(arguments, str):
        obj = arguments_object(arguments)
        return arguments if obj is not None else "{}"
    if isinstance(arguments, dict):
        return json.dumps(arguments, separators=(",", ":"))
    return "{}"


# ---------------------------------------------------------------------------
# compaction
# ---------------------------------------------------------------------------

def estimate_tokens(text: str, tokenizer=None) -> int:
    if not text:
        return 0
    if tokenizer is not None:
        return len(tokenizer.encode(text))
    return len(text) // 4 + 1


def message_tokens(m: dict, tokenizer=None) -> int:
    content = m.get("content") or ""
    if isinstance(content, list):  # multi-part content: count the text parts
        content = " ".join(p.get("text", "") for p in content if isinstance(p, dict))
    return estimate_tokens(content, tokenizer) + estimate_tokens(m.get("role", ""), tokenizer) + 3


def messages_tokens(messages: list[dict], tokenizer=None) -> int:
    return sum(message_tokens(m, tokenizer) for m in messages)


def compact_messages(messages: list[dict], budget: int, tokenizer=None) -> list[dict]:
    out = list(messages)

    def evict(pred):
        while messages_tokens(out, tokenizer) > budget:
            i = next((j for j, m in enumerate(out) if pred(m)), None)
            if i is None:
                return
            out.pop(i)

    if messages_tokens(out, tokenizer) <= budget:
        return out
    evict(lambda m: m.get("role") == "tool")
    evict(lambda m: m.get("role") != "system")
    return out
