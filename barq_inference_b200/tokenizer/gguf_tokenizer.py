"""Tokenizers built from GGUF metadata: SentencePiece-style BPE ("llama"), byte-level BPE ("gpt2"),
WordPiece ("bert") and Unigram ("t5").

Parity: ``GgufTokenizer`` (``vocab/src/gguf_tokenizer.rs:76-566``).  The reference tokenizes
SPM vocabularies with a greedy longest match (``tokenize_greedy``, ``:416-468``) and builds GPT-2 BPE by
writing temp files for an external crate.  Here both follow the published algorithms:

* SPM: text -> "▁"-joined symbols (one per UTF-8 character), repeatedly merge the adjacent pair whose
  concatenation is in the vocabulary with the highest score; unknown characters fall back to
  ``<0xNN>`` byte tokens.
* byte-level BPE: pre-tokenize with the GPT-2 / Llama-3 regex, map bytes to printable characters,
  merge by rank from ``tokenizer.ggml.merges``.
* WordPiece (BERT; the reference's ``WpmTokenizer`` returns "not yet implemented"): NFD, lower case,
  accents stripped, split on whitespace with punctuation and CJK characters as words of their own;
  each word, prefixed with "▁" (GGUF BERT vocabularies mark word starts that way instead of "##"
  continuations), is cut greedily into the longest vocabulary pieces; a word that cannot be covered
  becomes the unknown token.
* Unigram (T5 / SentencePiece unigram; the reference's ``UgmTokenizer`` is a stub): spaces become
  "▁" (plus a leading one), then a Viterbi pass picks the segmentation with the highest total
  score (log-probability) over the vocabulary; characters no piece covers cost the unknown
  token's score minus 10.

Special / control tokens written literally in the text are split out first and mapped directly.
"""
from __future__ import annotations

import heapq
import os
from dataclasses import dataclass, field
from functools import lru_cache

import regex

SPIECE = "▁"

# token_type values (ggml)
TT_NORMAL, TT_UNKNOWN, TT_CONTROL, TT_USER_DEFINED, TT_UNUSED, TT_BYTE = 1, 2, 3, 4, 5, 6

PRE_PATTERNS = {
    "gpt2": r"""'s|'t|'re|'ve|'m|'ll|'d| ?\p{L}+| ?\p{N}+| ?[^\s\p{L}\p{N}]+|\s+(?!\S)|\s+""",
    "llama3": r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+""",
    "qwen2": r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+""",
    "deepseek-llm": r"""[\r\n]|\s?\p{L}+|\s?\p{P}+|[一-龥ࠀ-一가-퟿]+|\p{N}+| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+""",
}
PRE_ALIASES = {"default": "gpt2", "llama-bpe": "llama3", "llama3": "llama3", "smaug-bpe": "llama3",
               "qwen2": "qwen2", "deepseek-llm": "deepseek-llm", "deepseek-v3": "llama3"}


@lru_cache(None)
def bytes_to_unicode() -> dict[int, str]:
    """The GPT-2 reversible byte -> printable character map."""
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + list(range(ord("®"), ord("ÿ") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return dict(zip(bs, map(chr, cs)))


@dataclass
class GGUFTokenizer:
    tokens: list[str]
    scores: list[float] = field(default_factory=list)
    token_types: list[int] = field(default_factory=list)
    merges: list[str] = field(default_factory=list)
    model: str = "llama"
    pre: str = "default"
    bos_id: int | None = 1
    eos_id: int | None = 2
    add_bos: bool = True
    add_space_prefix: bool = True

    def __post_init__(self):
        self.vocab = {t: i for i, t in enumerate(self.tokens)}
        if not self.token_types:
            self.token_types = [TT_NORMAL] * len(self.tokens)
        if not self.scores:
            self.scores = [0.0] * len(self.tokens)
        self.specials = sorted((t for t, ty in zip(self.tokens, self.token_types)
                                if ty in (TT_CONTROL, TT_USER_DEFINED) and t), key=len, reverse=True)
        self._special_re = regex.compile("(" + "|".join(regex.escape(s) for s in self.specials) + ")") if self.specials else None
        self.byte_tokens = {}
        for i, (t, ty) in enumerate(zip(self.tokens, self.token_types)):
            if ty == TT_BYTE or (len(t) == 6 and t.startswith("<0x") and t.endswith(">")):
                try:
                    self.byte_tokens[int(t[3:5], 16)] = i
                except ValueError:
                    pass
        self._native = _make_native(self)
        if self.model == "gpt2":
            self.ranks = {}
            for r, m in enumerate(self.merges):
                a, _, b = m.partition(" ")
                self.ranks[(a, b)] = r
            self.b2u = bytes_to_unicode()
            self.u2b = {v: k for k, v in self.b2u.items()}
            self.pre_re = regex.compile(PRE_PATTERNS[PRE_ALIASES.get(self.pre, "gpt2")])

    # ------------------------------------------------------------------ construction
    @staticmethod
    def from_metadata(md: dict) -> "GGUFTokenizer":
        toks = md.get("tokenizer.ggml.tokens")
        if toks is None:
            raise ValueError("GGUF has no tokenizer.ggml.tokens")
        toks = list(toks)
        model = str(md.get("tokenizer.ggml.model", "llama"))
        scores = md.get("tokenizer.ggml.scores")
        types = md.get("tokenizer.ggml.token_type")
        merges = md.get("tokenizer.ggml.merges")
        return GGUFTokenizer(
            tokens=toks,
            scores=[float(x) for x in scores] if scores is not None else [],
            token_types=[int(x) for x in types] if types is not None else [],
            merges=list(merges) if merges is not None else [],
            model=model if model in ("gpt2", "bert", "t5") else "llama",
            pre=str(md.get("tokenizer.ggml.pre", "default")),
            bos_id=md.get("tokenizer.ggml.bos_token_id"),
            eos_id=md.get("tokenizer.ggml.eos_token_id"),
            add_bos=bool(md.get("tokenizer.ggml.add_bos_token", model != "gpt2" or True)),
            add_space_prefix=bool(md.get("tokenizer.ggml.add_space_prefix", model != "gpt2")),
        )

    @property
    def vocab_size(self) -> int:
        return len(self.tokens)

    # ------------------------------------------------------------------ encode
    def encode(self, text: str, add_special: bool = True, parse_special: bool = True) -> list[int]:
        out: list[int] = []
        if add_special and self.add_bos and self.bos_id is not None:
            out.append(int(self.bos_id))
        pieces = self._special_re.split(text) if (parse_special and self._special_re) else [text]
        first = True
        for p in pieces:
            if not p:
                continue
            if parse_special and p in self.vocab and p in self.specials:
                out.append(self.vocab[p])
                first = False
                continue
            if self.model == "llama":
                out.extend(self._encode_spm(p, first))
            elif self.model == "bert":
                out.extend(self._encode_wpm(p))
            elif self.model == "t5":
                out.extend(self._encode_ugm(p, first))
            else:
                out.extend(self._encode_bpe(p))
            first = False
        return out

    def _encode_spm(self, text: str, first: bool) -> list[int]:
        if self.add_space_prefix and first and not text.startswith(" "):
            text = " " + text
        text = text.replace(" ", SPIECE)
        if self._native is not None:
            try:
                return self._native.spm(text)
            except UnicodeEncodeError:  # lone surrogates: not UTF-8 encodable, use the Python path
                pass
        return self._spm_py(text)

    def _spm_py(self, text: str) -> list[int]:
        syms = list(text)
        if not syms:
            return []
        # doubly linked list of symbols + heap of candidate merges ordered by (-score, position)
        prev = list(range(-1, len(syms) - 1))
        nxt = list(range(1, len(syms) + 1))
        nxt[-1] = -1
        alive = [True] * len(syms)
        heap: list[tuple[float, int, int, str]] = []

        def push(i: int):
            j = nxt[i]
            if j == -1:
                return
            cand = syms[i] + syms[j]
            tid = self.vocab.get(cand)
            if tid is not None:
                heapq.heappush(heap, (-self.scores[tid], i, j, cand))

        for i in range(len(syms) - 1):
            push(i)
        while heap:
            _, i, j, cand = heapq.heappop(heap)
            if not (alive[i] and alive[j]) or nxt[i] != j or syms[i] + syms[j] != cand:
                continue
            syms[i] = cand
            alive[j] = False
            nxt[i] = nxt[j]
            if nxt[j] != -1:
                prev[nxt[j]] = i
            if prev[i] != -1:
                push(prev[i])
            push(i)
        out = []
        i = 0
        while i != -1:
            s = syms[i]
            tid = self.vocab.get(s)
            if tid is not None:
                out.append(tid)
            else:
                for b in s.encode("utf-8"):
                    out.append(self.byte_tokens.get(b, self.vocab.get("<unk>", 0)))
            i = nxt[i]
        return out

    def _bpe_word(self, word: str) -> list[str]:
        parts = list(word)
        while len(parts) > 1:
            best, bi = None, -1
            for k in range(len(parts) - 1):
                r = self.ranks.get((parts[k], parts[k + 1]))
                if r is not None and (best is None or r < best):
                    best, bi = r, k
            if best is None:
                break
            parts[bi:bi + 2] = [parts[bi] + parts[bi + 1]]
        return parts

    def _encode_bpe(self, text: str) -> list[int]:
        if self._native is not None:
            words = ["".join(self.b2u[b] for b in m.encode("utf-8")) for m in self.pre_re.findall(text)]
            return self._native.bpe(words)
        return self._bpe_py(text)

    def _bpe_py(self, text: str) -> list[int]:
        out = []
        for m in self.pre_re.findall(text):
            word = "".join(self.b2u[b] for b in m.encode("utf-8"))
            if word in self.vocab:
                out.append(self.vocab[word])
                continue
            for p in self._bpe_word(word):
                tid = self.vocab.get(p)
                if tid is None:  # every single byte character is in a byte-level vocabulary
                    out.extend(self.vocab[c] for c in p if c in self.vocab)
                else:
                    out.append(tid)
        return out

    def _encode_wpm(self, text: str) -> list[int]:
        import unicodedata

        unk = self.vocab.get("[UNK]", self.vocab.get("<unk>", 0))
        norm = "".join(c for c in unicodedata.normalize("NFD", text.lower()) if unicodedata.category(c) != "Mn")
        words, cur = [], []
        for ch in norm:
            cp = ord(ch)
            if ch.isspace():
                if cur:
                    words.append("".join(cur))
                    cur = []
            elif unicodedata.category(ch).startswith("P") or (33 <= cp <= 47 or 58 <= cp <= 64 or 91 <= cp <= 96
                                                               or 123 <= cp <= 126) or _is_cjk(cp):
                if cur:
                    words.append("".join(cur))
                    cur = []
                words.append(ch)
            else:
                cur.append(ch)
        if cur:
            words.append("".join(cur))
        out: list[int] = []
        for w in words:
            w = SPIECE + w
            pieces, i, ok = [], 0, True
            while i < len(w):
                j = len(w)
                while j > i and w[i:j] not in self.vocab:
                    j -= 1
                if j == i:
                    ok = False
                    break
                pieces.append(self.vocab[w[i:j]])
                i = j
            out.extend(pieces if ok else [unk])
        return out

    def _encode_ugm(self, text: str, first: bool) -> list[int]:
        text = regex.sub(" +", " ", text)  # runs of spaces collapse (SentencePiece normalization)
        if self.add_space_prefix and first and not text.startswith(" "):
            text = " " + text
        text = text.replace(" ", SPIECE)
        n = len(text)
        if n == 0:
            return []
        unk = self.vocab.get("<unk>", self.vocab.get("[UNK]", 0))
        if not hasattr(self, "_ugm_maxlen"):
            self._ugm_maxlen = max((len(t) for t in self.tokens), default=1)
            normal = [sc for sc, ty in zip(self.scores, self.token_types) if ty == TT_NORMAL]
            self._ugm_unk_score = (min(normal) if normal else 0.0) - 10.0
        best = [float("-inf")] * (n + 1)
        back: list[tuple[int, int]] = [(0, -1)] * (n + 1)
        best[0] = 0.0
        for i in range(n):
            if best[i] == float("-inf"):
                continue
            covered = False
            for j in range(i + 1, min(n, i + self._ugm_maxlen) + 1):
                tid = self.vocab.get(text[i:j])
                if tid is None or self.token_types[tid] not in (TT_NORMAL, TT_USER_DEFINED):
                    continue
                covered = covered or j == i + 1
                sc = best[i] + (0.0 if self.token_types[tid] == TT_USER_DEFINED else self.scores[tid])
                if sc > best[j]:
                    best[j], back[j] = sc, (i, tid)
            if not covered:  # no single-character piece: this character costs the unknown token
                sc = best[i] + self._ugm_unk_score
                if sc > best[i + 1]:
                    best[i + 1], back[i + 1] = sc, (i, unk)
        out: list[int] = []
        j = n
        while j > 0:
            i, tid = back[j]
            out.append(tid)
            j = i
        out.reverse()
        merged: list[int] = []  # consecutive unknown characters collapse into one unknown token
        for t in out:
            if not (t == unk and merged and merged[-1] == unk):
                merged.append(t)
        return merged

    # ------------------------------------------------------------------ decode
    def token_bytes(self, tid: int) -> bytes:
        t = self.tokens[tid]
        ty = self.token_types[tid] if tid < len(self.token_types) else TT_NORMAL
        if ty == TT_CONTROL:
            return b""
        if self.model in ("llama", "bert", "t5"):
            if ty == TT_BYTE or (len(t) == 6 and t.startswith("<0x") and t.endswith(">")):
                try:
                    return bytes([int(t[3:5], 16)])
                except ValueError:
                    pass
            return t.replace(SPIECE, " ").encode("utf-8")
        if ty == TT_USER_DEFINED:
            return t.encode("utf-8")
        return bytes(self.u2b.get(c, ord("?") & 0xFF) for c in t)

    def decode(self, ids: list[int], skip_special: bool = True) -> str:
        buf = b"".join(self.token_bytes(i) for i in ids if 0 <= i < len(self.tokens))
        s = buf.decode("utf-8", errors="replace")
        if self.model in ("llama", "t5") and self.add_space_prefix and s.startswith(" "):
            s = s[1:]
        elif self.model == "bert" and s.startswith(" "):  # every word starts with "▁"
            s = s[1:]
        return s


class StreamDecoder:
    """Incremental detokenizer: emits text only once a full UTF-8 sequence is available."""

    def __init__(self, tok: GGUFTokenizer):
        self.tok = tok
        self.pending = b""
        self.first = True

    def push(self, tid: int) -> str:
        self.pending += self.tok.token_bytes(tid)
        try:
            s = self.pending.decode("utf-8")
        except UnicodeDecodeError as e:
            if e.reason == "unexpected end of data":
                return ""
            s = self.pending.decode("utf-8", errors="replace")
        self.pending = b""
        return s

    def flush(self) -> str:
        s = self.pending.decode("utf-8", errors="replace")
        self.pending = b""
        return s


def _is_cjk(cp: int) -> bool:
    return (0x4E00 <= cp <= 0x9FFF or 0x3400 <= cp <= 0x4DBF or 0x20000 <= cp <= 0x2A6DF or 0x2A700 <= cp <= 0x2B73F
            or 0x2B740 <= cp <= 0x2B81F or 0x2B820 <= cp <= 0x2CEAF or 0xF900 <= cp <= 0xFAFF
            or 0x2F800 <= cp <= 0x2FA1F)


def _make_native(tok: "GGUFTokenizer"):
    """The C++ merge loops (``_native.NativeTokenizer``) for this vocabulary, or None when the
    extension is not built or ``BARQ_NATIVE_TOKENIZER=0``."""
    if os.environ.get("BARQ_NATIVE_TOKENIZER", "1") == "0":
        return None
    try:
        import torch  # noqa: F401  (loads the libraries the extension links against)

        from .. import _native
    except ImportError:
        return None
    byte_ids = [tok.byte_tokens.get(b, -1) for b in range(256)]
    try:
        return _native.NativeTokenizer(list(tok.tokens), [float(x) for x in tok.scores], list(tok.merges) if tok.model == "gpt2" else [],
                                       byte_ids, int(tok.vocab.get("<unk>", 0)))
    except (UnicodeError, TypeError):
        return None


def synthetic_tokenizer(vocab: int, seed: int = 0) -> GGUFTokenizer:
    """A deterministic SPM-style vocabulary for random-init models (bytes, letters, common bigrams)."""
    toks = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    types = [TT_UNKNOWN, TT_CONTROL, TT_CONTROL] + [TT_BYTE] * 256
    base = [SPIECE] + [chr(c) for c in range(ord("a"), ord("z") + 1)] + [chr(c) for c in range(ord("A"), ord("Z") + 1)]
    base += list("0123456789.,!?;:'\"()-")
    words = ["the", "and", "of", "to", "in", "is", "it", "that", "for", "on", "with", "as", "was", "barq", "model",
             "token", "fast", "gpu", "hello", "world", "json", "true", "false", "null"]
    extra = []
    for w in words:  # every prefix, so score-ordered pair merges can reach the whole word
        for k in range(2, len(w) + 1):
            extra += [SPIECE + w[:k], w[:k]]
        extra.append(SPIECE + w[0])
    seen = set(toks)
    for t in base + extra:
        if t not in seen:
            toks.append(t)
            types.append(TT_NORMAL)
            seen.add(t)
    letters = [chr(c) for c in range(ord("a"), ord("z") + 1)]
    i = 0
    while len(toks) < vocab:
        a, b = letters[i % 26], letters[(i // 26) % 26]
        t = (SPIECE if (i // 676) % 2 else "") + a + b + ("" if i < 1352 else letters[(i // 1352) % 26])
        if t not in seen:
            toks.append(t)
            types.append(TT_NORMAL)
            seen.add(t)
        else:
            toks.append(f"<extra_{len(toks)}>")
            types.append(TT_UNUSED)
        i += 1
    toks = toks[:vocab]
    types = types[:vocab]
    scores = [-float(i) / 100.0 for i in range(len(toks))]
    return GGUFTokenizer(tokens=toks, scores=scores, token_types=types, model="llama")
