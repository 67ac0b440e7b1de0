"""Host-side sampler chain (CPU, PyTorch) for the rarely used samplers and for the CPU engine.

Parity: the reference's sampler set (``sampling/src/lib.rs:54-65``, ``penalties.rs:7-442``):
greedy, distribution, temperature, top-k, top-p, min-p, typical, Mirostat v1/v2, XTC and the
repetition / frequency / presence penalties.  The reference's Mirostat, typical and XTC bodies do
not implement the published algorithms (its Mirostat rescales logits by mu/tau, its "typical"
thresholds raw probabilities); these follow the papers:

* Mirostat v1 / v2: Basu et al., "Mirostat: a neural text decoding algorithm that directly controls
  perplexity" (ICLR 2021) — target surprise tau, learning rate eta, mu initialised to 2*tau.
* Locally typical sampling: Meister et al., "Locally Typical Sampling" (TACL 2022).
* XTC ("exclude top choices"): with probability ``xtc_probability``, drop every token whose
  probability exceeds ``xtc_threshold`` except the least likely of them.

The common chain (penalties, temperature, top-k, top-p, min-p) runs on the GPU in the fused sampler
kernel; sequences that ask for Mirostat, typical or XTC are sampled on the host from their logits
row: by the C++ chain ``_native.HostSampler`` (``csrc/native/sampler_native.cpp``: partial sorts
instead of whole-row sorts) when the extension is built, else by :class:`HostSampler` here, which is
also that chain's oracle.
"""
from __future__ import annotations

import math

import torch


def apply_penalties(logits: torch.Tensor, history: list[int], repetition: float, frequency: float,
                    presence: float) -> torch.Tensor:
    if not history or (repetition == 1.0 and frequency == 0.0 and presence == 0.0):
        return logits
    ids, counts = torch.unique(torch.tensor(history, dtype=torch.long), return_counts=True)
    ids, counts = ids[ids < logits.numel()], counts[ids < logits.numel()]
    lg = logits.clone()
    v = lg[ids]
    if repetition != 1.0:
        v = torch.where(v > 0, v / repetition, v * repetition)
    v = v - counts.float() * frequency - presence
    lg[ids] = v
    return lg


def top_k_filter(logits: torch.Tensor, k: int) -> torch.Tensor:
    if k <= 0 or k >= logits.numel():
        return logits
    th = torch.topk(logits, k).values[-1]
    return logits.masked_fill(logits < th, -math.inf)


def top_p_filter(logits: torch.Tensor, p: float, min_keep: int = 1) -> torch.Tensor:
    if p >= 1.0:
        return logits
    sl, si = torch.sort(logits, descending=True)
    probs = torch.softmax(sl, -1)
    cum = probs.cumsum(-1)
    remove = cum - probs >= p
    remove[:min_keep] = False
    out = logits.clone()
    out[si[remove]] = -math.inf
    return out


def min_p_filter(logits: torch.Tensor, p: float) -> torch.Tensor:
    if p <= 0.0:
        return logits
    probs = torch.softmax(logits, -1)
    return logits.masked_fill(probs < p * probs.max(), -math.inf)


def typical_filter(logits: torch.Tensor, p: float, min_keep: int = 1) -> torch.Tensor:
    """Keep the tokens whose surprise is closest to the distribution's entropy until mass >= p."""
    if p >= 1.0:
        return logits
    logp = torch.log_softmax(logits, -1)
    probs = logp.exp()
    ent = -(probs * torch.nan_to_num(logp, neginf=0.0)).sum()
    shifted = (-logp - ent).abs()
    order = torch.argsort(shifted)
    cum = probs[order].cumsum(-1)
    n_keep = max(min_keep, int((cum < p).sum().item()) + 1)
    out = torch.full_like(logits, -math.inf)
    keep = order[:n_keep]
    out[keep] = logits[keep]
    return out


def xtc_filter(logits: torch.Tensor, probability: float, threshold: float, gen: torch.Generator) -> torch.Tensor:
    if probability <= 0.0 or torch.rand((), generator=gen).item() >= probability:
        return logits
    probs = torch.softmax(logits, -1)
    above = (probs > threshold).nonzero().flatten()
    if above.numel() < 2:
        return logits
    keep = above[torch.argmin(probs[above])]
    out = logits.clone()
    drop = above[above != keep]
    out[drop] = -math.inf
    return out


class HostSampler:
    """Per-sequence sampler state (Mirostat's mu, the RNG)."""

    def __init__(self, params, vocab: int):
        self.p = params
        self.vocab = vocab
        self.gen = torch.Generator().manual_seed(int(params.seed) if params.seed else 0x5EED)
        self.mu = 2.0 * params.mirostat_tau

    def sample(self, logits: torch.Tensor, seq=None) -> int:
        p = self.p
        lg = logits.float().reshape(-1)[: self.vocab]
        if seq is not None and p.needs_penalties:
            hist = seq.tokens[-p.penalty_last_n:] if p.penalty_last_n > 0 else []
            lg = apply_penalties(lg, hist, p.repetition_penalty, p.frequency_penalty, p.presence_penalty)
        if p.temperature <= 0.0:
            return int(torch.argmax(lg))
        if p.mirostat == 1:
            return self._mirostat_v1(lg / p.temperature)
        if p.mirostat == 2:
            return self._mirostat_v2(lg / p.temperature)
        lg = top_k_filter(lg / p.temperature, p.top_k)
        lg = typical_filter(lg, p.typical_p)
        lg = top_p_filter(lg, p.top_p)
        lg = min_p_filter(lg, p.min_p)
        lg = xtc_filter(lg, p.xtc_probability, p.xtc_threshold, self.gen)
        probs = torch.softmax(lg, -1)
        return int(torch.multinomial(probs, 1, generator=self.gen))

    def _mirostat_v1(self, lg: torch.Tensor, m: int = 100) -> int:
        p = self.p
        sl, si = torch.sort(lg, descending=True)
        probs = torch.softmax(sl, -1)
        n = min(m, probs.numel() - 1)
        # estimate the Zipf exponent s from the top-m probabilities
        i = torch.arange(1, n, dtype=torch.float64)
        t = torch.log((i + 1) / i)
        b = torch.log(probs[:n - 1].double() / probs[1:n].double())
        s_hat = float((t * b).sum() / (t * t).sum())
        eps = s_hat - 1
        N = probs.numel()
        k = ((eps * 2 ** self.mu) / (1 - N ** (-eps))) ** (1 / s_hat) if eps > 0 else N
        k = int(max(1, min(N, round(k))))
        pk = torch.softmax(sl[:k], -1)
        j = int(torch.multinomial(pk, 1, generator=self.gen))
        surprise = -math.log2(max(1e-30, float(probs[j])))
        self.mu -= p.mirostat_eta * (surprise - p.mirostat_tau)
        return int(si[j])

    def _mirostat_v2(self, lg: torch.Tensor) -> int:
        p = self.p
        sl, si = torch.sort(lg, descending=True)
        probs = torch.softmax(sl, -1)
        surprise = -torch.log2(probs.clamp_min(1e-30))
        keep = int((surprise <= self.mu).sum().item())
        keep = max(1, keep)
        pk = torch.softmax(sl[:keep], -1)
        j = int(torch.multinomial(pk, 1, generator=self.gen))
        s = -math.log2(max(1e-30, float(pk[j])))
        self.mu -= p.mirostat_eta * (s - p.mirostat_tau)
        return int(si[j])


def sample_chain(logits: torch.Tensor, params, history: list[int], gen: torch.Generator) -> int:
    """Stateless full chain (used by the CPU engine for the common samplers)."""
    p = params
    lg = logits.float().reshape(-1)
    if p.needs_penalties:
        hist = history[-p.penalty_last_n:] if p.penalty_last_n > 0 else []
        lg = apply_penalties(lg, hist, p.repetition_penalty, p.frequency_penalty, p.presence_penalty)
    if p.temperature <= 0.0:
        return int(torch.argmax(lg))
    lg = top_k_filter(lg / p.temperature, p.top_k)
    lg = top_p_filter(lg, p.top_p)
    lg = min_p_filter(lg, p.min_p)
    probs = torch.softmax(lg, -1)
    return int(torch.multinomial(probs, 1, generator=gen))


class NativeHostSampler:
    """:class:`HostSampler` on the C++ chain (same filters and Mirostat updates; its own RNG)."""

    def __init__(self, params, vocab: int):
        from .. import _native

        p = self.p = params
        self.vocab = vocab
        self.impl = _native.HostSampler(
            vocab=vocab, seed=int(p.seed) if p.seed else 0x5EED, temperature=p.temperature, top_k=p.top_k,
            top_p=p.top_p, min_p=p.min_p, typical_p=p.typical_p, repetition=p.repetition_penalty,
            frequency=p.frequency_penalty, presence=p.presence_penalty, mirostat=p.mirostat, tau=p.mirostat_tau,
            eta=p.mirostat_eta, xtc_probability=p.xtc_probability, xtc_threshold=p.xtc_threshold)

    @property
    def mu(self) -> float:
        return self.impl.mu

    def _history(self, seq) -> list[int]:
        p = self.p
        if seq is None or not p.needs_penalties or p.penalty_last_n <= 0:
            return []
        return seq.last_tokens(p.penalty_last_n)

    def sample(self, logits: torch.Tensor, seq=None) -> int:
        return self.impl.sample(logits.detach().float().reshape(-1).cpu().numpy(), self._history(seq))

    def distribution(self, logits: torch.Tensor, seq=None) -> tuple[list[int], list[float]]:
        """The kept tokens and the probabilities the next draw uses (XTC, being random, left out)."""
        return self.impl.distribution(logits.detach().float().reshape(-1).cpu().numpy(), self._history(seq))


def new_host_sampler(params, vocab: int):
    """The C++ chain when ``_native`` is built (``BARQ_NATIVE_SAMPLER=0`` forces the Python one)."""
    import os

    if os.environ.get("BARQ_NATIVE_SAMPLER", "1") != "0":
        try:
            from .. import _native

            if hasattr(_native, "HostSampler"):
                return NativeHostSampler(params, vocab)
        except ImportError:
            pass
    return HostSampler(params, vocab)
