"""The C++ host sampler chain (``_native.HostSampler``) against the Python chain in
``sampling/host_samplers.py``: the same kept tokens and final distribution for every filter
combination (penalties, temperature, top-k, typical, top-p, min-p), the same Mirostat v1 / v2
truncation and mu updates, XTC's exclusion rule, and sample frequencies that follow the
distribution."""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from barq_inference_b200.engine.sampling_params import SamplingParams  # noqa: E402
from barq_inference_b200.sampling import host_samplers as hs  # noqa: E402

try:
    from barq_inference_b200 import _native
except ImportError:  # pragma: no cover
    _native = None
pytestmark = pytest.mark.skipif(_native is None or not hasattr(_native, "HostSampler"),
                                reason="native extension not built")


class _Seq:
    def __init__(self, toks):
        self.toks = toks

    @property
    def tokens(self):
        return self.toks

    def last_tokens(self, n):
        return self.toks[-n:]


def _python_distribution(lg, p, hist):
    """The Python chain up to the draw (XTC off): (kept ids, probabilities)."""
    x = lg.float().clone()
    if p.needs_penalties and hist:
        x = hs.apply_penalties(x, hist[-p.penalty_last_n:], p.repetition_penalty, p.frequency_penalty,
                               p.presence_penalty)
    x = hs.top_k_filter(x / p.temperature, p.top_k)
    x = hs.typical_filter(x, p.typical_p)
    x = hs.top_p_filter(x, p.top_p)
    x = hs.min_p_filter(x, p.min_p)
    probs = torch.softmax(x, -1)
    ids = torch.nonzero(x > -math.inf).flatten()
    return ids.tolist(), probs[ids].double().numpy()


CASES = [dict(temperature=0.8, top_k=40), dict(temperature=1.0, top_p=0.9), dict(temperature=1.3, typical_p=0.5),
         dict(temperature=0.7, min_p=0.05), dict(temperature=1.0, top_k=200, typical_p=0.9, top_p=0.95, min_p=0.01),
         dict(temperature=1.1, typical_p=0.2, repetition_penalty=1.3, frequency_penalty=0.2, presence_penalty=0.4),
         dict(temperature=0.9, top_p=0.5, top_k=3)]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("vocab", [50, 4096, 32000])
def test_native_chain_keeps_the_same_tokens(case, vocab):
    g = torch.Generator().manual_seed(case * 31 + vocab)
    p = SamplingParams(**CASES[case])
    nat = hs.NativeHostSampler(p, vocab)
    for trial in range(4):
        lg = torch.randn(vocab, generator=g) * (1 + 2 * trial)  # flat to peaked
        seq = _Seq(torch.randint(0, vocab, (80,), generator=g).tolist())
        ids, probs = nat.distribution(lg, seq)
        want_ids, want_p = _python_distribution(lg, p, seq.tokens)
        assert sorted(ids) == want_ids
        got = dict(zip(ids, probs))
        np.testing.assert_allclose([got[i] for i in want_ids], want_p, rtol=1e-4, atol=1e-7)


def test_native_sample_frequencies_follow_the_distribution():
    vocab = 64
    g = torch.Generator().manual_seed(5)
    lg = torch.randn(vocab, generator=g) * 1.5
    p = SamplingParams(temperature=1.0, top_k=10, typical_p=0.95, seed=3)
    nat = hs.NativeHostSampler(p, vocab)
    ids, probs = nat.distribution(lg)
    n = 40000
    counts = np.bincount([nat.sample(lg) for _ in range(n)], minlength=vocab)
    assert set(np.nonzero(counts)[0].tolist()) <= set(ids)
    for i, q in zip(ids, probs):  # each count within 5 standard deviations of its expectation
        assert abs(counts[i] - n * q) <= 5 * math.sqrt(n * q * (1 - q)) + 1, (i, counts[i], n * q)
    # the same seed gives the same stream; greedy ignores the RNG
    a, b = hs.NativeHostSampler(p, vocab), hs.NativeHostSampler(p, vocab)
    assert [a.sample(lg) for _ in range(50)] == [b.sample(lg) for _ in range(50)]
    gr = hs.NativeHostSampler(SamplingParams(temperature=0.0, mirostat=2), vocab)
    assert gr.sample(lg) == int(lg.argmax())


@pytest.mark.parametrize("mirostat", [1, 2])
@pytest.mark.parametrize("vocab", [300, 32000])
def test_native_mirostat_matches_the_python_truncation_and_update(mirostat, vocab):
    """Same truncation set at the current mu, and mu moves by eta * (surprise - tau) of the drawn
    token, where the surprise is measured under the full (v1) or truncated (v2) distribution."""
    g = torch.Generator().manual_seed(vocab + mirostat)
    p = SamplingParams(temperature=1.0, mirostat=mirostat, mirostat_tau=3.0, mirostat_eta=0.2, seed=9)
    nat = hs.NativeHostSampler(p, vocab)
    py = hs.HostSampler(p, vocab)
    for step in range(30):
        lg = torch.randn(vocab, generator=g) * (0.5 + step % 4)
        py.mu = nat.mu
        ids, probs = nat.distribution(lg)
        # the Python truncation at this mu: replay its arithmetic
        sl, si = torch.sort(lg.float(), descending=True)
        full = torch.softmax(sl, -1)
        if mirostat == 1:
            n = min(100, vocab - 1)
            i = torch.arange(1, n, dtype=torch.float64)
            t = torch.log((i + 1) / i)
            b = torch.log(full[:n - 1].double() / full[1:n].double())
            s_hat = float((t * b).sum() / (t * t).sum())
            eps = s_hat - 1
            k = ((eps * 2 ** py.mu) / (1 - vocab ** (-eps))) ** (1 / s_hat) if eps > 0 else vocab
            k = int(max(1, min(vocab, round(k))))
        else:
            k = max(1, int((-torch.log2(full.clamp_min(1e-30)) <= py.mu).sum()))
        assert len(ids) == k and set(ids) == set(si[:k].tolist())  # tied logits may swap places
        want = dict(zip(si[:k].tolist(), torch.softmax(sl[:k], -1).double().tolist()))
        np.testing.assert_allclose(probs, [want[i] for i in ids], rtol=1e-4, atol=1e-8)
        mu0 = nat.mu
        tok = nat.sample(lg)
        j = ids.index(tok)
        q = float(torch.softmax(lg.float(), -1)[tok]) if mirostat == 1 else probs[j]
        assert nat.mu == pytest.approx(mu0 - 0.2 * (-math.log2(max(1e-30, q)) - 3.0), rel=1e-5, abs=1e-6)


def test_native_xtc_excludes_all_but_the_least_likely_top_choice():
    vocab = 100
    lg = torch.full((vocab,), -10.0)
    lg[[3, 7, 11]] = torch.tensor([3.0, 2.5, 2.0])  # three tokens above a 0.1 threshold
    p = SamplingParams(temperature=1.0, xtc_probability=1.0, xtc_threshold=0.1, seed=4)
    nat = hs.NativeHostSampler(p, vocab)
    draws = [nat.sample(lg) for _ in range(300)]
    assert 3 not in draws and 7 not in draws and draws.count(11) > 250
    off = hs.NativeHostSampler(SamplingParams(temperature=1.0, xtc_probability=0.0, seed=4), vocab)
    assert 3 in [off.sample(lg) for _ in range(100)]


def test_factory_and_argument_checks(monkeypatch):
    p = SamplingParams(temperature=1.0, mirostat=2)
    assert isinstance(hs.new_host_sampler(p, 10), hs.NativeHostSampler)
    monkeypatch.setenv("BARQ_NATIVE_SAMPLER", "0")
    assert isinstance(hs.new_host_sampler(p, 10), hs.HostSampler)
    with pytest.raises(ValueError):
        hs.NativeHostSampler(p, 10).sample(torch.randn(5))  # shorter than the vocabulary
