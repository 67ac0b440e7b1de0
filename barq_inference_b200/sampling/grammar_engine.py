"""Glue between requests and the grammar matcher: per-engine token strings / trie, per-request state.

The matcher is the native recognizer (``_native.NativeMatcher``, C++) when the extension is built,
else the Python ``GrammarMatcher``; both expose ``allowed_mask`` / ``allowed_ids`` / ``accept`` /
``done``.  ``BARQ_NATIVE_GRAMMAR=0`` forces the Python one.
"""
from __future__ import annotations

import os

from .grammar import CharClass, Grammar, GrammarMatcher, TokenTrie
from .json_mode import JSON_GBNF, schema_to_gbnf

_CACHE_ATTR = "_grammar_cache"


def token_strings(tokenizer, vocab: int) -> list[str | None]:
    out: list[str | None] = []
    for tid in range(vocab):
        if tokenizer is None or tid >= tokenizer.vocab_size:
            out.append(None)
            continue
        try:
            s = tokenizer.token_bytes(tid).decode("utf-8")
        except UnicodeDecodeError:
            s = None
        out.append(s or None)
    return out


def _native_mod():
    if os.environ.get("BARQ_NATIVE_GRAMMAR", "1") == "0":
        return None
    try:
        import torch  # noqa: F401  (loads the libraries the extension links against)

        from .. import _native
    except ImportError:
        return None
    return _native


def native_rules(g: Grammar) -> list:
    """The parsed grammar as plain lists for the native recognizer."""
    out = []
    for rule in g.rules:
        alts = []
        for alt in rule:
            alts.append([("c", [tuple(r) for r in el.ranges], bool(el.negated)) if isinstance(el, CharClass)
                         else ("r", int(el.rule)) for el in alt])
        out.append(alts)
    return out


def make_grammar_state(engine, params):
    text = params.grammar
    if text is None and params.json_schema is not None:
        text = schema_to_gbnf(params.json_schema)
    elif text is None:
        text = JSON_GBNF
    cache = engine.__dict__.setdefault(_CACHE_ATTR, {})
    if "strings" not in cache:
        tok = getattr(engine, "tokenizer", None)
        if tok is None:  # without token strings every token would be disallowed
            raise ValueError("grammar / JSON-mode sampling needs the engine's tokenizer (engine.tokenizer)")
        cache["strings"] = token_strings(tok, engine.cfg.vocab)
    nat = _native_mod()
    if nat is not None:
        if "ntrie" not in cache:
            cache["ntrie"] = nat.NativeTrie(cache["strings"])
        ng = cache.get(("ng", text))
        if ng is None:
            g = Grammar(text)
            ng = nat.NativeGrammar(native_rules(g), g.root)
            cache[("ng", text)] = ng
        return nat.NativeMatcher(ng, cache["ntrie"], [int(e) for e in engine.cfg.eos_ids])
    if "trie" not in cache:
        cache["trie"] = TokenTrie(cache["strings"])
    g = cache.get(("g", text))
    if g is None:
        g = Grammar(text)
        cache[("g", text)] = g
        cache[("m", text)] = {}
    return GrammarMatcher(g, cache["trie"], engine.cfg.vocab, tuple(engine.cfg.eos_ids), cache["strings"],
                          cache[("m", text)])
