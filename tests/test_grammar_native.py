"""Native (C++) grammar recognizer == the Python recognizer: same allowed-token sets step by step
along JSON documents and custom GBNF grammars, same completion state, same bitmasks."""
import random

import numpy as np
import pytest
import torch  # noqa: F401  (the extension links against torch)

from barq_inference_b200.sampling.grammar import Grammar, GrammarMatcher, TokenTrie
from barq_inference_b200.sampling.grammar_engine import native_rules, token_strings
from barq_inference_b200.sampling.json_mode import JSON_GBNF, schema_to_gbnf
from barq_inference_b200.tokenizer.gguf_tokenizer import synthetic_tokenizer

nat = pytest.importorskip("barq_inference_b200._native")

TOK = synthetic_tokenizer(4000)
STRS = token_strings(TOK, 4000)
BY_STR = {}
for _i, _s in enumerate(STRS):
    if _s is not None:
        BY_STR.setdefault(_s, _i)


def _pair(text):
    g = Grammar(text)
    py_m = GrammarMatcher(g, TokenTrie(STRS), 4000, (2,), STRS, {})
    n = nat.NativeMatcher(nat.NativeGrammar(native_rules(g), g.root), nat.NativeTrie(STRS), [2])
    return py_m, n


def _walk(text, doc, rng):
    """Feed ``doc`` token by token (random allowed tokens where the doc allows) comparing masks."""
    py_m, n = _pair(text)
    steps = 0
    for ch in doc:
        a, b = sorted(set(py_m.allowed_ids())), sorted(set(n.allowed_ids()))
        assert a == b, (doc, steps)
        assert np.array_equal(py_m.allowed_mask(125), n.allowed_mask(125))
        tid = BY_STR.get(ch)
        if tid is None or tid not in a:
            break
        py_m.accept(tid)
        n.accept(tid)
        assert py_m.done() == n.done()
        steps += 1
    return steps


@pytest.mark.parametrize("doc", ['{"a": [1, 2, {"b": "xy"}], "c": true}', '{"k": [null, false, -1.5e3]}', ' {"s": "str"} '])
def test_json_grammar_masks_match(doc):
    assert _walk(JSON_GBNF, doc, random.Random(0)) > 3


def test_random_token_walks_match():
    gram = 'root ::= item ("," item)*\nitem ::= [a-z]+ | "(" root ")" | [0-9]{1,3}\n'
    for seed in range(5):
        rng = random.Random(seed)
        py_m, n = _pair(gram)
        for _ in range(25):
            a = sorted(set(py_m.allowed_ids()))
            assert a == sorted(set(n.allowed_ids()))
            if not a:
                break
            tid = rng.choice(a)
            py_m.accept(tid)
            n.accept(tid)
            assert py_m.done() == n.done()
            if tid == 2:
                break


def test_schema_grammar_and_engine_state():
    from types import SimpleNamespace

    from barq_inference_b200.engine.sampling_params import SamplingParams
    from barq_inference_b200.sampling.grammar_engine import make_grammar_state

    schema = {"type": "object", "properties": {"name": {"type": "string"}, "n": {"type": "integer"}},
              "required": ["name", "n"]}
    assert _walk(schema_to_gbnf(schema), '{"name": "ab", "n": 12}', random.Random(1)) > 5
    eng = SimpleNamespace(tokenizer=TOK, cfg=SimpleNamespace(vocab=4000, eos_ids=(2,)))
    st = make_grammar_state(eng, SamplingParams(json_mode=True))
    assert type(st).__name__ == "NativeMatcher" and st.allowed_mask(125).shape == (125,)


@pytest.mark.parametrize("text,want", [("12x", True), ("1x", False), ("12345x", False), ("1234xaaa", True),
                                       ("123x", True), ("12", False)])
def test_bounded_repetition(text, want):
    g = Grammar('root ::= [0-9]{2,4} "x"{1} [a]{0,}\n')
    assert Grammar.complete(g.accept_text(g.initial(), text)) == want
