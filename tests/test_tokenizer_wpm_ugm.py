"""WordPiece (BERT) and Unigram (T5) tokenizers from GGUF-style vocabularies (CPU)."""
import itertools

from barq_inference_b200.tokenizer.gguf_tokenizer import TT_CONTROL, TT_NORMAL, TT_UNKNOWN, GGUFTokenizer


def _wpm():
    toks = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "▁hello", "▁world", "▁un", "aff", "able", "▁", ",", "▁,", "▁!",
            "▁中", "▁x", "y", "▁cafe"]
    types = [TT_CONTROL, TT_UNKNOWN, TT_CONTROL, TT_CONTROL] + [TT_NORMAL] * (len(toks) - 4)
    return GGUFTokenizer(tokens=toks, token_types=types, model="bert", bos_id=2, eos_id=3, add_bos=True)


def test_wordpiece_greedy_longest_match():
    t = _wpm()
    v = t.vocab
    assert t.encode("Hello  WORLD", add_special=False) == [v["▁hello"], v["▁world"]]
    assert t.encode("unaffable", add_special=False) == [v["▁un"], v["aff"], v["able"]]
    assert t.encode("hello, world!", add_special=False) == [v["▁hello"], v["▁,"], v["▁world"], v["▁!"]]
    assert t.encode("zzz hello", add_special=False) == [v["[UNK]"], v["▁hello"]]  # uncoverable word
    assert t.encode("Café", add_special=False) == [v["▁cafe"]]  # accents stripped
    assert t.encode("中", add_special=True) == [2, v["▁中"]]
    assert t.decode(t.encode("hello world", add_special=False)) == "hello world"


def _ugm():
    toks = ["<pad>", "</s>", "<unk>", "▁", "▁a", "b", "ab", "▁ab", "c", "bc", "a", "▁abc"]
    scores = [0, 0, 0, -1.0, -2.0, -2.5, -2.0, -3.5, -2.0, -1.5, -2.2, -9.0]
    types = [TT_CONTROL, TT_CONTROL, TT_UNKNOWN] + [TT_NORMAL] * (len(toks) - 3)
    return GGUFTokenizer(tokens=toks, scores=scores, token_types=types, model="t5", bos_id=None, eos_id=1,
                         add_bos=False)


def _brute(t, text):
    """Best-scoring segmentation by enumerating every cut (the Viterbi pass must find it)."""
    best, arg = float("-inf"), None
    n = len(text)
    for mask in itertools.product([0, 1], repeat=n - 1):
        cuts = [0] + [i + 1 for i, m in enumerate(mask) if m] + [n]
        pieces = [text[a:b] for a, b in zip(cuts, cuts[1:])]
        if all(p in t.vocab and t.token_types[t.vocab[p]] == TT_NORMAL for p in pieces):
            sc = sum(t.scores[t.vocab[p]] for p in pieces)
            if sc > best:
                best, arg = sc, [t.vocab[p] for p in pieces]
    return arg


def test_unigram_viterbi_is_optimal():
    t = _ugm()
    for s in ["abc", "ab abc", "abcabc", "a b", "bcab", "cab ab"]:
        norm = ("▁" + s).replace(" ", "▁")
        assert t.encode(s, add_special=False) == _brute(t, norm), s
    ids = t.encode("ab  zz", add_special=False)  # collapsed spaces; uncovered chars -> one <unk>
    assert ids.count(t.vocab["<unk>"]) == 1
    assert t.decode(t.encode("ab abc", add_special=False)) == "ab abc"


def test_from_metadata_selects_model():
    md = {"tokenizer.ggml.model": "bert", "tokenizer.ggml.tokens": ["[UNK]", "▁a"], "tokenizer.ggml.token_type": [2, 1]}
    assert GGUFTokenizer.from_metadata(md).model == "bert"
    md["tokenizer.ggml.model"] = "t5"
    assert GGUFTokenizer.from_metadata(md).model == "t5"
