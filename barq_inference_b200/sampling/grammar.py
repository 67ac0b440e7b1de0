"""GBNF grammars: parser, incremental pushdown recognizer and per-step token masks.

Parity: ``GrammarParser`` / ``Grammar`` / ``GrammarRule`` (``barq_core/src/grammar/parser.rs:13-101``,
``grammar/mod.rs:45-54``) and ``GrammarSampler`` (``sampling/src/grammar_sampler.rs:20-320``).  The
reference applies a fixed root-rule mask and never advances its rule stack (``accept_token`` only
counts); here the grammar state advances with every accepted token, so constrained output is valid.

Grammar model: each rule is a list of alternatives, each alternative a sequence of elements —
a character class (set of code-point ranges, optionally negated) or a reference to another rule.
Repetition (``*``, ``+``, ``?``) and parenthesised groups are desugared into generated rules.
A parse state is a set of stacks; a stack is a tuple of (rule, alternative, position) frames whose
top frame points at the next expected terminal.  An empty stack means the input so far is a
complete sentence.

Token masks walk a trie of the vocabulary's token strings with the current state set and prune
dead branches; masks are memoised per state set, which keeps structured formats such as JSON fast.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


class GrammarError(ValueError):
    pass


@dataclass(frozen=True)
class CharClass:
    ranges: tuple[tuple[int, int], ...]
    negated: bool = False

    def match(self, c: int) -> bool:
        hit = any(a <= c <= b for a, b in self.ranges)
        return hit != self.negated


@dataclass(frozen=True)
class RuleRef:
    rule: int


# ------------------------------------------------------------------ parser

class _Parser:
    def __init__(self, text: str):
        self.s = text
        self.i = 0
        self.names: dict[str, int] = {}
        self.rules: list[list[list]] = []

    def rule_id(self, name: str) -> int:
        if name not in self.names:
            self.names[name] = len(self.rules)
            self.rules.append([])
        return self.names[name]

    def new_rule(self, alts) -> int:
        rid = len(self.rules)
        self.names[f"__gen{rid}"] = rid
        self.rules.append(alts)
        return rid

    def ws(self, newlines: bool = True):
        while self.i < len(self.s):
            c = self.s[self.i]
            if c == "#":
                while self.i < len(self.s) and self.s[self.i] != "\n":
                    self.i += 1
            elif c in " \t\r" or (newlines and c == "\n"):
                self.i += 1
            else:
                break

    def name(self) -> str:
        j = self.i
        while self.i < len(self.s) and (self.s[self.i].isalnum() or self.s[self.i] in "-_"):
            self.i += 1
        if j == self.i:
            raise GrammarError(f"expected a rule name at {j}")
        return self.s[j:self.i]

    def char(self) -> int:
        c = self.s[self.i]
        if c != "\\":
            self.i += 1
            return ord(c)
        self.i += 1
        e = self.s[self.i]
        self.i += 1
        simple = {"n": 10, "t": 9, "r": 13, "\\": 92, '"': 34, "[": 91, "]": 93, "-": 45, "/": 47, "b": 8, "f": 12}
        if e in simple:
            return simple[e]
        if e in "xuU":
            n = {"x": 2, "u": 4, "U": 8}[e]
            v = int(self.s[self.i:self.i + n], 16)
            self.i += n
            return v
        return ord(e)

    def parse(self) -> tuple[list, dict]:
        self.ws()
        while self.i < len(self.s):
            nm = self.name()
            self.ws()
            if not self.s.startswith("::=", self.i):
                raise GrammarError(f"expected ::= after {nm!r}")
            self.i += 3
            alts = self.alternatives(nested=False)
            rid = self.rule_id(nm)
            self.rules[rid] = alts
            self.ws()
        for n, rid in self.names.items():
            if not self.rules[rid] and not n.startswith("__gen"):
                raise GrammarError(f"undefined rule {n!r}")
        if "root" not in self.names:
            raise GrammarError("grammar has no 'root' rule")
        return self.rules, self.names

    def alternatives(self, nested: bool) -> list:
        alts = [self.sequence(nested)]
        while self.i < len(self.s) and self.s[self.i] == "|":
            self.i += 1
            alts.append(self.sequence(nested))
        return alts

    def sequence(self, nested: bool) -> list:
        seq = []
        while True:
            self.ws(newlines=nested)
            if self.i >= len(self.s):
                break
            c = self.s[self.i]
            if c == "\n" or c == "|" or c == ")":
                break
            # lookahead: a new rule definition starts on this line
            j = self.i
            if c.isalpha():
                k = j
                while k < len(self.s) and (self.s[k].isalnum() or self.s[k] in "-_"):
                    k += 1
                k2 = k
                while k2 < len(self.s) and self.s[k2] in " \t":
                    k2 += 1
                if self.s.startswith("::=", k2):
                    break
            start = len(seq)
            if c == '"':
                self.i += 1
                while self.s[self.i] != '"':
                    v = self.char()
                    seq.append(CharClass(((v, v),)))
                self.i += 1
            elif c == "[":
                self.i += 1
                neg = False
                if self.s[self.i] == "^":
                    neg = True
                    self.i += 1
                ranges = []
                while self.s[self.i] != "]":
                    a = self.char()
                    b = a
                    if self.s[self.i] == "-" and self.s[self.i + 1] != "]":
                        self.i += 1
                        b = self.char()
                    ranges.append((a, b))
                self.i += 1
                seq.append(CharClass(tuple(ranges), neg))
            elif c == ".":
                self.i += 1
                seq.append(CharClass(((0, 0x10FFFF),)))
            elif c == "(":
                self.i += 1
                alts = self.alternatives(nested=True)
                self.ws()
                if self.i >= len(self.s) or self.s[self.i] != ")":
                    raise GrammarError("unbalanced parenthesis")
                self.i += 1
                seq.append(RuleRef(self.new_rule(alts)))
            elif c.isalpha():
                seq.append(RuleRef(self.rule_id(self.name())))
            else:
                raise GrammarError(f"unexpected {c!r} at {self.i}")
            # repetition operators apply to the last element
            if self.i < len(self.s) and self.s[self.i] in "*+?":
                op = self.s[self.i]
                self.i += 1
                last = seq[start:]
                del seq[start:]
                if op == "?":
                    seq.append(RuleRef(self.new_rule([last, []])))
                else:
                    rid = self.new_rule([])
                    self.rules[rid] = [last + [RuleRef(rid)], []]
                    if op == "*":
                        seq.append(RuleRef(rid))
                    else:
                        seq.extend(last + [RuleRef(rid)])
            elif self.i < len(self.s) and self.s[self.i] == "{":
                # bounded repetition {m}, {m,}, {m,n}: m copies, then a star rule or n-m nested optionals
                close = self.s.find("}", self.i)
                if close < 0:
                    raise GrammarError("unterminated repetition count")
                body = self.s[self.i + 1: close].replace(" ", "")
                self.i = close + 1
                try:
                    if "," in body:
                        lo_s, hi_s = body.split(",", 1)
                        lo, hi = int(lo_s), (int(hi_s) if hi_s else None)
                    else:
                        lo = hi = int(body)
                except ValueError:
                    raise GrammarError(f"bad repetition count {{{body}}}") from None
                if lo < 0 or (hi is not None and hi < lo):
                    raise GrammarError(f"bad repetition count {{{body}}}")
                last = seq[start:]
                del seq[start:]
                for _ in range(lo):
                    seq.extend(last)
                if hi is None:
                    rid = self.new_rule([])
                    self.rules[rid] = [last + [RuleRef(rid)], []]
                    seq.append(RuleRef(rid))
                elif hi > lo:
                    tail: list = []
                    for _ in range(hi - lo):  # R ::= last R_prev | (empty)
                        tail = [RuleRef(self.new_rule([last + tail, []]))]
                    seq.extend(tail)
        return seq


# ------------------------------------------------------------------ recognizer

class Grammar:
    def __init__(self, text: str, root: str = "root"):
        self.rules, self.names = _Parser(text).parse()
        self.root = self.names[root]
        self._expand_cache: dict = {}

    def _expand(self, stack: tuple) -> frozenset:
        """All stacks reachable from `stack` whose top points at a terminal (or that are empty)."""
        hit = self._expand_cache.get(stack)
        if hit is not None:
            return hit
        out = set()
        todo = [stack]
        seen = set()
        while todo:
            st = todo.pop()
            if st in seen:
                continue
            seen.add(st)
            if not st:
                out.add(st)
                continue
            r, a, p = st[-1]
            alt = self.rules[r][a]
            if p >= len(alt):
                todo.append(st[:-1])
                continue
            el = alt[p]
            if isinstance(el, CharClass):
                out.add(st)
                continue
            base = st[:-1] + ((r, a, p + 1),)
            for ai in range(len(self.rules[el.rule])):
                todo.append(base + ((el.rule, ai, 0),))
        res = frozenset(out)
        if len(self._expand_cache) < 200000:
            self._expand_cache[stack] = res
        return res

    def initial(self) -> frozenset:
        out = set()
        for ai in range(len(self.rules[self.root])):
            out |= self._expand(((self.root, ai, 0),))
        return frozenset(out)

    def step(self, stacks: frozenset, c: int) -> frozenset:
        out = set()
        for st in stacks:
            if not st:
                continue
            r, a, p = st[-1]
            el = self.rules[r][a][p]
            if el.match(c):
                out |= self._expand(st[:-1] + ((r, a, p + 1),))
        return frozenset(out)

    def accept_text(self, stacks: frozenset, text: str) -> frozenset:
        for ch in text:
            stacks = self.step(stacks, ord(ch))
            if not stacks:
                break
        return stacks

    @staticmethod
    def complete(stacks: frozenset) -> bool:
        return any(len(st) == 0 for st in stacks)

    @staticmethod
    def can_continue(stacks: frozenset) -> bool:
        return any(len(st) > 0 for st in stacks)


class TokenTrie:
    """Prefix tree over the vocabulary's token strings (tokens whose bytes are not valid UTF-8 on
    their own are left out of constrained generation)."""

    def __init__(self, token_strings: list[str | None]):
        self.children: list[dict[str, int]] = [{}]
        self.tokens_at: list[list[int]] = [[]]
        for tid, s in enumerate(token_strings):
            if not s:
                continue
            node = 0
            for ch in s:
                nxt = self.children[node].get(ch)
                if nxt is None:
                    nxt = len(self.children)
                    self.children[node][ch] = nxt
                    self.children.append({})
                    self.tokens_at.append([])
                node = nxt
            self.tokens_at[node].append(tid)


class GrammarMatcher:
    """Per-request grammar state: allowed-token bitmask for the next step, then ``accept``."""

    def __init__(self, grammar: Grammar, trie: TokenTrie, vocab: int, eos_ids: tuple[int, ...],
                 token_strings: list[str | None], mask_cache: dict | None = None):
        self.g = grammar
        self.trie = trie
        self.vocab = vocab
        self.eos_ids = eos_ids
        self.tok = token_strings
        self.stacks = grammar.initial()
        self.cache = mask_cache if mask_cache is not None else {}

    def allowed_ids(self) -> list[int]:
        key = self.stacks
        hit = self.cache.get(key)
        if hit is not None:
            return hit
        allowed: list[int] = []
        g = self.g
        todo = [(0, self.stacks)]
        while todo:
            node, st = todo.pop()
            for ch, child in self.trie.children[node].items():
                nst = g.step(st, ord(ch))
                if not nst:
                    continue
                allowed.extend(self.trie.tokens_at[child])
                todo.append((child, nst))
        if Grammar.complete(self.stacks):
            allowed.extend(self.eos_ids)
        if len(self.cache) < 4096:
            self.cache[key] = allowed
        return allowed

    def allowed_mask(self, words: int) -> np.ndarray:
        m = np.zeros(words * 32, dtype=bool)
        ids = self.allowed_ids()
        if not ids:  # dead end: let the model finish instead of emitting garbage
            ids = list(self.eos_ids)
        m[np.asarray(ids, dtype=np.int64)] = True
        # bit i of word w allows token 32*w + i
        weights = (np.uint64(1) << np.arange(32, dtype=np.uint64))
        return (m.reshape(-1, 32).astype(np.uint64) * weights).sum(1).astype(np.uint32)

    def accept(self, tid: int) -> None:
        if tid in self.eos_ids:
            self.stacks = frozenset()
            return
        s = self.tok[tid] if tid < len(self.tok) else None
        if s:
            self.stacks = self.g.accept_text(self.stacks, s)

    def done(self) -> bool:
        return not Grammar.can_continue(self.stacks)
