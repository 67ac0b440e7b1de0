"""JSON mode: the JSON GBNF grammar and JSON-schema -> GBNF conversion, plus output validation.

Parity: ``json_mode`` (``sampling/src/json_mode/mod.rs:17-130``: ``json_object_gbnf``,
``schema_to_gbnf`` over a ``JsonSchema`` enum, ``validate_output``).  Used by ``--json`` in the CLI
and by ``response_format: {"type": "json_object" | "json_schema"}`` in the HTTP API.
"""
from __future__ import annotations

import json
import re

JSON_GBNF = r'''
root   ::= ws object ws
value  ::= object | array | string | number | ("true" | "false" | "null")
object ::= "{" ws ( string ws ":" ws value ( ws "," ws string ws ":" ws value )* )? ws "}"
array  ::= "[" ws ( value ( ws "," ws value )* )? ws "]"
string ::= "\"" ( [^"\\\x00-\x1f] | "\\" ( ["\\/bfnrt] | "u" [0-9a-fA-F] [0-9a-fA-F] [0-9a-fA-F] [0-9a-fA-F] ) )* "\""
number ::= "-"? ( "0" | [1-9] [0-9]* ) ( "." [0-9]+ )? ( [eE] [-+]? [0-9]+ )?
ws     ::= [ \t\n]*
'''

JSON_ARRAY_GBNF = JSON_GBNF.replace("root   ::= ws object ws", "root   ::= ws array ws")

_PRIMS = {
    "string": 'string', "number": 'number', "integer": 'integer', "boolean": '("true" | "false")',
    "null": '"null"',
}
_BASE = r'''
value  ::= object | array | string | number | ("true" | "false" | "null")
object ::= "{" ws ( string ws ":" ws value ( ws "," ws string ws ":" ws value )* )? ws "}"
array  ::= "[" ws ( value ( ws "," ws value )* )? ws "]"
string ::= "\"" ( [^"\\\x00-\x1f] | "\\" ( ["\\/bfnrt] | "u" [0-9a-fA-F] [0-9a-fA-F] [0-9a-fA-F] [0-9a-fA-F] ) )* "\""
number ::= "-"? ( "0" | [1-9] [0-9]* ) ( "." [0-9]+ )? ( [eE] [-+]? [0-9]+ )?
integer ::= "-"? ( "0" | [1-9] [0-9]* )
ws     ::= [ \t\n]*
'''


def _lit(s: str) -> str:
    """GBNF string literal matching exactly the characters of ``s``."""
    out = []
    for ch in s:
        if ch in '"\\':
            out.append("\\" + ch)
        elif ch == "\n":
            out.append("\\n")
        elif ord(ch) < 32:
            out.append("\\x%02x" % ord(ch))
        else:
            out.append(ch)
    return '"' + "".join(out) + '"'


class _SchemaConv:
    def __init__(self):
        self.rules: dict[str, str] = {}
        self.n = 0

    def add(self, body: str, hint: str = "r") -> str:
        self.n += 1
        name = f"{re.sub('[^a-zA-Z0-9]', '-', hint)}-{self.n}"
        self.rules[name] = body
        return name

    def visit(self, sch: dict, hint: str = "r") -> str:
        if not isinstance(sch, dict) or not sch:
            return "value"
        if "enum" in sch:
            return self.add(" | ".join(_lit(json.dumps(v)) for v in sch["enum"]), hint)
        if "const" in sch:
            return self.add(_lit(json.dumps(sch["const"])), hint)
        for key in ("anyOf", "oneOf"):
            if key in sch:
                return self.add(" | ".join(self.visit(s, hint) for s in sch[key]), hint)
        t = sch.get("type")
        if isinstance(t, list):
            return self.add(" | ".join(self.visit({**sch, "type": x}, hint) for x in t), hint)
        if t == "object" or "properties" in sch:
            props = sch.get("properties", {})
            req = set(sch.get("required", list(props)))
            parts = []
            first = True
            for k, v in props.items():
                r = self.visit(v, k)
                kv = f'{_lit(json.dumps(k))} ws ":" ws {r}'
                if k in req:
                    parts.append(kv if first else f'ws "," ws {kv}')
                    first = False
                else:
                    sep = "" if first else 'ws "," ws '
                    parts.append("( " + sep + kv + " )?")
            if not props:
                return "object"
            return self.add('"{" ws ' + " ".join(parts) + ' ws "}"', hint)
        if t == "array":
            it = self.visit(sch.get("items", {}), hint + "-item")
            mn = int(sch.get("minItems", 0))
            if mn > 0:
                return self.add(f'"[" ws {it} ( ws "," ws {it} )* ws "]"', hint)
            return self.add(f'"[" ws ( {it} ( ws "," ws {it} )* )? ws "]"', hint)
        if t in _PRIMS:
            return _PRIMS[t]
        return "value"


def schema_to_gbnf(schema: dict) -> str:
    c = _SchemaConv()
    root = c.visit(schema, "root")
    lines = [f"root ::= ws {root} ws"] + [f"{k} ::= {v}" for k, v in c.rules.items()]
    return "\n".join(lines) + "\n" + _BASE


def validate_output(text: str) -> bool:
    try:
        json.loads(text)
        return True
    except (ValueError, TypeError):
        return False
