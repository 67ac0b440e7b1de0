"""Speculative decoding's device-side pieces on CPU tensors: batched sampling distributions (same
filters as the host samplers) and the rejection step (greedy prefix rule; sampled output follows
the target distribution)."""
import torch

from barq_inference_b200.engine.sampling_params import SamplingParams
from barq_inference_b200.engine.speculative import _probs, verify_drafts
from barq_inference_b200.sampling.host_samplers import min_p_filter, top_k_filter, top_p_filter


def test_batched_probs_match_host_filters():
    g = torch.Generator().manual_seed(0)
    lg = torch.randn(5, 300, generator=g) * 3
    for kw in (dict(temperature=0.7, top_k=20), dict(temperature=1.0, top_p=0.8),
               dict(temperature=1.3, min_p=0.05), dict(temperature=0.9, top_k=50, top_p=0.9, min_p=0.02)):
        p = SamplingParams(**kw)
        got = _probs(lg, p)
        for i in range(lg.shape[0]):
            x = top_k_filter(lg[i] / p.temperature, p.top_k)
            x = top_p_filter(x, p.top_p)
            x = min_p_filter(x, p.min_p)
            assert torch.allclose(got[i], torch.softmax(x, -1), atol=1e-6), kw
    one = _probs(lg, SamplingParams(temperature=0.0))
    assert torch.equal(one.argmax(-1), lg.argmax(-1)) and torch.equal(one.sum(-1), torch.ones(5))


def test_verify_greedy_prefix_rule():
    V, k = 10, 3
    ps = torch.zeros(k + 1, V)
    for i, t in enumerate([4, 7, 2, 9]):
        ps[i, t] = 1.0
    qs = torch.full((k, V), 0.1)
    n, new = verify_drafts(ps, qs, torch.tensor([4, 7, 5]), greedy=True)
    assert n == 2 and new == [4, 7, 2]
    n, new = verify_drafts(ps, qs, torch.tensor([4, 7, 2]), greedy=True)
    assert n == 3 and new == [4, 7, 2, 9]  # all accepted: bonus token from the last row
    n, new = verify_drafts(ps, qs, torch.tensor([1, 7, 2]), greedy=True)
    assert n == 0 and new == [4]


def test_verify_sampled_output_follows_target():
    """Draft x ~ q, then the rejection step: the first emitted token is distributed as p."""
    p = torch.tensor([0.5, 0.2, 0.15, 0.1, 0.05])
    q = torch.tensor([0.1, 0.4, 0.1, 0.3, 0.1])
    gen = torch.Generator().manual_seed(3)
    ps = torch.stack([p, p])
    qs = q[None]
    counts = torch.zeros(5)
    n = 6000
    for _ in range(n):
        x = torch.multinomial(q, 1, generator=gen)
        _, new = verify_drafts(ps, qs, x, greedy=False, gen=gen)
        counts[new[0]] += 1
    assert (counts / n - p).abs().max() < 0.025, counts / n


def test_one_hot_drafts_keep_the_target_distribution():
    """Prompt-lookup drafts are deterministic (q one-hot at the proposed token x): accepting x with
    probability p(x) and otherwise sampling norm(max(0, p - q)) must give exactly p."""
    import torch

    from barq_inference_b200.engine.speculative import verify_drafts

    p = torch.tensor([[0.5, 0.2, 0.2, 0.1], [0.25, 0.25, 0.25, 0.25]])
    q = torch.zeros(1, 4)
    q[0, 1] = 1.0  # the draft proposes token 1
    g = torch.Generator().manual_seed(0)
    counts = torch.zeros(4)
    n = 20000
    for _ in range(n):
        n_acc, toks = verify_drafts(p, q, torch.tensor([1]), False, g)
        counts[toks[0]] += 1
    assert torch.allclose(counts / n, p[0], atol=0.015), counts / n
