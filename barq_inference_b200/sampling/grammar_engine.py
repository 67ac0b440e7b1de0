"""Glue between requests and the grammar matcher: per-engine token strings / trie, per-request state."""
from __future__ import annotations

from .grammar import Grammar, GrammarMatcher, TokenTrie
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


def make_grammar_state(engine, params) -> GrammarMatcher:
    text = params.grammar
    if text is None and params.json_schema is not None:
        text = schema_to_gbnf(params.json_schema)
    elif text is None:
        text = JSON_GBNF
    cache = engine.__dict__.setdefault(_CACHE_ATTR, {})
    if "trie" not in cache:
        tok = getattr(engine, "tokenizer", None)
        cache["strings"] = token_strings(tok, engine.cfg.vocab)
        cache["trie"] = TokenTrie(cache["strings"])
    g = cache.get(("g", text))
    if g is None:
        g = Grammar(text)
        cache[("g", text)] = g
        cache[("m", text)] = {}
    return GrammarMatcher(g, cache["trie"], engine.cfg.vocab, tuple(engine.cfg.eos_ids), cache["strings"],
                          cache[("m", text)])
