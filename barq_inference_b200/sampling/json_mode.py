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
string ::= "\"" char* "\""
char   ::= [^"\\\x00-\x1f] | "\\" ( ["\\/bfnrt] | "u" [0-9a-fA-F] [0-9a-fA-F] [0-9a-fA-F] [0-9a-fA-F] )
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
    """JSON schema -> GBNF rules.  Supported: type (incl. lists), enum, const, anyOf / oneOf, allOf
    (object schemas merged), properties / required (required ones first, then optional ones in
    schema order, commas always well placed), items with minItems / maxItems, string minLength /
    maxLength, nested objects and arrays, local ``$ref`` into ``$defs`` / ``definitions`` (recursive
    schemas become recursive rules).  Anything else falls back to any JSON value."""

    def __init__(self, root: dict | None = None):
        self.rules: dict[str, str] = {}
        self.n = 0
        self.root = root or {}
        self.refs: dict[str, str] = {}

    def add(self, body: str, hint: str = "r") -> str:
        self.n += 1
        name = f"{re.sub('[^a-zA-Z0-9]', '-', hint)}-{self.n}"
        self.rules[name] = body
        return name

    def _ref(self, ref: str) -> str:
        if ref in self.refs:
            return self.refs[ref]
        if not ref.startswith("#/"):
            return "value"  # remote references are not fetched
        node = self.root
        for part in ref[2:].split("/"):
            node = node.get(part.replace("~1", "/").replace("~0", "~"), {}) if isinstance(node, dict) else {}
        name = self.add("value", "ref-" + ref.rsplit("/", 1)[-1])  # placeholder: recursion resolves to it
        self.refs[ref] = name
        self.rules[name] = self.visit(node, "def-" + ref.rsplit("/", 1)[-1])
        return name

    @staticmethod
    def _merge_all_of(sch: dict) -> dict:
        out = {k: v for k, v in sch.items() if k != "allOf"}
        props, req = dict(out.get("properties", {})), list(out.get("required", []))
        for sub in sch["allOf"]:
            if isinstance(sub, dict):
                props.update(sub.get("properties", {}))
                req += [r for r in sub.get("required", []) if r not in req]
                for k, v in sub.items():
                    if k not in ("properties", "required"):
                        out.setdefault(k, v)
        if props:
            out["properties"] = props
            out["type"] = out.get("type", "object")
        if req:
            out["required"] = req
        return out

    def _object(self, sch: dict, hint: str) -> str:
        props = sch.get("properties", {})
        if not props:
            return "object"
        req = [k for k in props if k in set(sch.get("required", []))]
        opt = [k for k in props if k not in req]
        kv = {k: f'{_lit(json.dumps(k))} ws ":" ws {self.visit(props[k], k)}' for k in props}
        if req:
            body = ' ws "," ws '.join(kv[k] for k in req)
            body += "".join(f' ( ws "," ws {kv[k]} )?' for k in opt)
        else:
            # any in-order subset of the optional properties, comma separated: start at any of them,
            # then each later one may follow after a comma
            tails: dict[int, str] = {}
            for i in range(len(opt) - 1, -1, -1):
                nxt = "".join(f' ( ws "," ws {kv[opt[j]]} )?' for j in range(i + 1, len(opt)))
                tails[i] = kv[opt[i]] + nxt
            body = "( " + " | ".join(f"( {tails[i]} )" for i in range(len(opt))) + " )?"
        return self.add('"{" ws ' + body + ' ws "}"', hint)

    def _array(self, sch: dict, hint: str) -> str:
        it = self.visit(sch.get("items", {}), hint + "-item")
        mn = max(0, int(sch.get("minItems", 0)))
        mx = sch.get("maxItems")
        mx = None if mx is None else max(int(mx), 0)
        if mx == 0:
            return self.add('"[" ws "]"', hint)
        rest_lo = max(mn - 1, 0)
        rest = f"{{{rest_lo},}}" if mx is None else f"{{{rest_lo},{mx - 1}}}"
        inner = f'{it} ( ws "," ws {it} ){rest}'
        body = f'"[" ws {inner} ws "]"' if mn > 0 else f'"[" ws ( {inner} )? ws "]"'
        return self.add(body, hint)

    def _string(self, sch: dict, hint: str) -> str:
        lo, hi = sch.get("minLength"), sch.get("maxLength")
        if lo is None and hi is None:
            return "string"
        lo = max(0, int(lo or 0))
        rep = f"{{{lo},}}" if hi is None else f"{{{lo},{max(int(hi), lo)}}}"
        return self.add(f'"\\"" char{rep} "\\""', hint)

    def visit(self, sch: dict, hint: str = "r") -> str:
        if not isinstance(sch, dict) or not sch:
            return "value"
        if "$ref" in sch:
            return self._ref(str(sch["$ref"]))
        if "allOf" in sch:
            return self.visit(self._merge_all_of(sch), hint)
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
            return self._object(sch, hint)
        if t == "array":
            return self._array(sch, hint)
        if t == "string":
            return self._string(sch, hint)
        if t in _PRIMS:
            return _PRIMS[t]
        return "value"


def schema_to_gbnf(schema: dict) -> str:
    c = _SchemaConv(schema)
    root = c.visit(schema, "root")
    lines = [f"root ::= ws {root} ws"] + [f"{k} ::= {v}" for k, v in c.rules.items()]
    return "\n".join(lines) + "\n" + _BASE


def validate_output(text: str) -> bool:
    try:
        json.loads(text)
        return True
    except (ValueError, TypeError):
        return False
