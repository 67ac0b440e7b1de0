"""Chat-side request handling shared by the OpenAI HTTP server and the UDS server: normalization of
chat messages (tool results, earlier assistant tool calls) and OpenAI ``tools`` / ``tool_choice``
(a system prompt describing the functions, a JSON schema that constrains a required call, and the
recognition of a function-call reply)."""
from __future__ import annotations

import json
from typing import Any


def normalize_messages(messages: Any) -> list[dict]:
    """OpenAI chat messages -> {role, content} turns for the chat template: a tool's result becomes a
    user turn, an assistant turn that called a tool carries the call as JSON text."""
    if not isinstance(messages, list) or not messages:
        raise ValueError("messages must be a non-empty list")
    msgs = []
    for m in messages:
        if not isinstance(m, dict) or ("content" not in m and "tool_calls" not in m):
            raise ValueError("each message needs role and content")
        m = dict(m)
        if m.get("content") is None and m.get("tool_calls"):  # an earlier assistant tool call
            m["content"] = json.dumps([c.get("function", c) for c in m["tool_calls"]])
        if m.get("role") == "tool":  # a tool's result goes back to the model as a user turn
            m = {"role": "user", "content": f"Tool result ({m.get('name') or m.get('tool_call_id', 'tool')}): "
                                            f"{m.get('content', '')}"}
        m["content"] = m.get("content") or ""
        msgs.append(m)
    return msgs


def tool_setup(body: dict) -> dict | None:
    """OpenAI ``tools`` / ``tool_choice``: a system prompt describing the functions, and (when a call
    is required or a function is named) a JSON schema that constrains the reply to
    ``{"name": ..., "arguments": {...}}`` for one of them."""
    tools = body.get("tools")
    if not tools:
        return None
    if not isinstance(tools, list):
        raise ValueError("tools must be a list")
    fns = []
    for t in tools:
        f = t.get("function", t) if isinstance(t, dict) else None
        if not isinstance(f, dict) or not f.get("name"):
            raise ValueError("each tool needs a function with a name")
        fns.append(f)
    choice = body.get("tool_choice", "auto")
    if choice == "none":
        return None
    if isinstance(choice, dict):
        name = (choice.get("function") or {}).get("name")
        fns_c = [f for f in fns if f["name"] == name]
        if not fns_c:
            raise ValueError(f"tool_choice names an unknown function {name!r}")
    else:
        fns_c = fns
    forced = choice == "required" or isinstance(choice, dict)
    schema = None
    if forced:
        alts = [{"type": "object", "properties": {"name": {"const": f["name"]},
                                                  "arguments": f.get("parameters") or {"type": "object"}},
                 "required": ["name", "arguments"]} for f in fns_c]
        schema = alts[0] if len(alts) == 1 else {"anyOf": alts}
    desc = json.dumps([{"name": f["name"], "description": f.get("description", ""),
                        "parameters": f.get("parameters", {})} for f in fns])
    prompt = ("You can call these functions. To call one, reply with only a JSON object "
              '{"name": <function name>, "arguments": <arguments object>}.\nFunctions: ' + desc)
    return {"prompt": prompt, "schema": schema, "names": {f["name"] for f in fns}}


def tool_call_of(text: str, names: set) -> dict | None:
    """{"name", "arguments"} when ``text`` is a call of one of the functions ``names``, else None."""
    try:
        obj = json.loads(text)
    except ValueError:
        return None
    if isinstance(obj, dict) and obj.get("name") in names and isinstance(obj.get("arguments"), dict):
        return {"name": obj["name"], "arguments": obj["arguments"]}
    return None


def tool_names(body: dict) -> set:
    return {(t.get("function", t) or {}).get("name") for t in body.get("tools") or [] if isinstance(t, dict)}
