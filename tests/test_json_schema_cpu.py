"""JSON schema -> GBNF: the grammar accepts valid instances and rejects invalid ones (CPU)."""
import json

import pytest

from barq_inference_b200.sampling.grammar import Grammar
from barq_inference_b200.sampling.json_mode import schema_to_gbnf


def accepts(schema, doc: str) -> bool:
    g = Grammar(schema_to_gbnf(schema))
    return Grammar.complete(g.accept_text(g.initial(), doc))


OBJ = {"type": "object", "properties": {"a": {"type": "integer"}, "b": {"type": "string"},
                                        "c": {"type": "boolean"}}, "required": ["b"]}


@pytest.mark.parametrize("doc,ok", [
    ('{"b": "x"}', True), ('{"b": "x", "a": 1}', True), ('{"b": "x", "a": 1, "c": true}', True),
    ('{"b": "x", "c": false}', True), ('{"a": 1}', False), ('{, "b": "x"}', False), ('{"b": 1}', False),
])
def test_required_and_optional_properties(doc, ok):
    assert accepts(OBJ, doc) == ok


@pytest.mark.parametrize("doc,ok", [('{}', True), ('{"x": 1}', True), ('{"y": "s"}', True), ('{"x": 1, "y": "s"}', True),
                                    ('{, "y": "s"}', False), ('{"y": "s", "x": 1}', False)])
def test_all_optional_properties(doc, ok):
    sch = {"type": "object", "properties": {"x": {"type": "integer"}, "y": {"type": "string"}}, "required": []}
    assert accepts(sch, doc) == ok


def test_arrays_strings_refs_allof():
    arr = {"type": "array", "items": {"type": "integer"}, "minItems": 2, "maxItems": 3}
    assert [accepts(arr, d) for d in ("[1]", "[1, 2]", "[1,2,3]", "[1,2,3,4]", "[]")] == [False, True, True, False, False]
    s = {"type": "string", "minLength": 2, "maxLength": 3}
    assert [accepts(s, json.dumps(x)) for x in ("a", "ab", "abc", "abcd")] == [False, True, True, False]
    tree = {"$defs": {"node": {"type": "object", "properties": {"v": {"type": "integer"},
                                                                "kids": {"type": "array", "items": {"$ref": "#/$defs/node"}}},
                               "required": ["v"]}},
            "$ref": "#/$defs/node"}
    assert accepts(tree, '{"v": 1, "kids": [{"v": 2}, {"v": 3, "kids": []}]}')
    assert not accepts(tree, '{"kids": []}')
    both = {"allOf": [{"type": "object", "properties": {"p": {"type": "integer"}}, "required": ["p"]},
                      {"properties": {"q": {"type": "string"}}, "required": ["q"]}]}
    assert accepts(both, '{"p": 1, "q": "z"}') and not accepts(both, '{"p": 1}')
    assert accepts({"enum": ["red", 3, None]}, "null") and not accepts({"enum": ["red"]}, '"blue"')
