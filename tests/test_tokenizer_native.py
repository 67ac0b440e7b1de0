"""Native (C++) tokenizer merge loops == the Python implementation, for SPM score merges and GPT-2
byte-level BPE rank merges, on random multilingual text."""
import collections
import random

import pytest
import torch  # noqa: F401  (the extension links against torch)

from barq_inference_b200.tokenizer.gguf_tokenizer import GGUFTokenizer, bytes_to_unicode, synthetic_tokenizer

pytest.importorskip("barq_inference_b200._native")

ALPHABET = list("abcdefghijklmnopqrstuvwxyz      ABCXYZ0123456789.,!?'\"-\n\t") + ["é", "ü", "ß", "中", "文", "😀", "▁"]


def _texts(n, seed):
    rng = random.Random(seed)
    words = ["the", "model", "hello", "world", "json", "barq", "token", "fast", "gpu", "and"]
    out = []
    for _ in range(n):
        parts = []
        for _ in range(rng.randint(1, 30)):
            parts.append(rng.choice(words) if rng.random() < 0.5 else
                         "".join(rng.choice(ALPHABET) for _ in range(rng.randint(1, 8))))
        out.append(rng.choice(["", " ", "  "]).join(parts) if rng.random() < 0.3 else " ".join(parts))
    return out


def test_spm_native_matches_python():
    tok = synthetic_tokenizer(3000)
    assert tok._native is not None
    for t in _texts(300, 0) + ["", " ", "▁▁", "hello world", "<s>hi</s>"]:
        for first in (True, False):
            text = (" " + t if tok.add_space_prefix and first and not t.startswith(" ") else t).replace(" ", "▁")
            assert tok._native.spm(text) == tok._spm_py(text), repr(t)
        assert tok.encode(t) == tok.encode(t)  # stable


def _train_bpe(corpus, n_merges):
    """A small byte-level BPE (most frequent pair first) to get a realistic merge list."""
    b2u = bytes_to_unicode()
    words = collections.Counter("".join(b2u[b] for b in w.encode("utf-8")) for t in corpus for w in t.split(" "))
    seqs = {w: list(w) for w in words}
    merges = []
    for _ in range(n_merges):
        pairs = collections.Counter()
        for w, c in words.items():
            s = seqs[w]
            for a, b in zip(s, s[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        (a, b), _ = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))
        merges.append(f"{a} {b}")
        for w in seqs:
            s, i, out = seqs[w], 0, []
            while i < len(s):
                if i + 1 < len(s) and s[i] == a and s[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(s[i])
                    i += 1
            seqs[w] = out
    toks = sorted(set(b2u.values())) + [m.replace(" ", "") for m in merges]
    toks = list(dict.fromkeys(toks))
    return toks, merges


def test_bpe_native_matches_python():
    toks, merges = _train_bpe(_texts(200, 1), 300)
    tok = GGUFTokenizer(tokens=toks, merges=merges, model="gpt2", pre="llama-bpe", add_bos=False, bos_id=None)
    assert tok._native is not None
    for t in _texts(300, 2) + ["", "hello world", "😀😀 中文", "  leading"]:
        assert tok._encode_bpe(t) == tok._bpe_py(t), repr(t)
    ids = tok.encode("hello world, the model is fast")
    assert tok.decode(ids) == "hello world, the model is fast"
