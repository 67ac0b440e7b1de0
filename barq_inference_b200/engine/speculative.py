"""Speculative decoding: a draft model proposes k tokens, the target verifies them in ONE batched
forward, and standard rejection sampling keeps the output distribution equal to the target's.

Parity: ``SpeculativeEngine`` (``advanced/src/speculative.rs:113-334``: draft k = speculation_steps,
verify, accept on match, stats) and the dead ``models/src/speculative_{decode,engine}.rs`` (presets
code / creative / max_speed, draft pairing).  The reference verifies token by token with one target
call per drafted token and a "simplified" probability ratio; here the target scores all k drafted
positions in a single forward over the paged KV cache and acceptance follows Leviathan et al.,
"Fast Inference from Transformers via Speculative Decoding" (ICML 2023): accept draft token x with
probability min(1, p(x)/q(x)), otherwise sample from norm(max(0, p - q)); if all k are accepted, one
bonus token is sampled from p.  Greedy requests (temperature 0) accept exactly the prefix where the
target's argmax agrees, so their output is identical to plain greedy decoding.
"""
from __future__ import annotations

import time
from dataclasses import dataclass

import torch

from ..models.runner import StepInput
from .sampling_params import SamplingParams


@dataclass
class SpeculativeConfig:
    draft_max: int = 4
    draft_min: int = 1
    adaptive: bool = True  # shrink/grow k with the running acceptance rate

    @staticmethod
    def preset(name: str, draft_max: int | None = None) -> "SpeculativeConfig":
        base = {"default": SpeculativeConfig(4), "code": SpeculativeConfig(8), "creative": SpeculativeConfig(3),
                "max_speed": SpeculativeConfig(12)}[name or "default"]
        if draft_max:
            base.draft_max = int(draft_max)
        return base


@dataclass
class SpecStats:
    drafted: int = 0
    accepted: int = 0
    steps: int = 0
    bonus: int = 0

    @property
    def acceptance_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0


@dataclass
class SpecResult:
    tokens: list[int]
    acceptance_rate: float
    stats: SpecStats
    elapsed_s: float = 0.0
    finish_reason: str = "length"


class _Seq:
    """One sequence's paged-KV state inside an engine, driven directly through its runner."""

    def __init__(self, engine):
        self.e = engine
        self.table: list[int] = []
        self.len = 0  # tokens whose K/V are valid

    def ensure(self, n_tokens: int):
        self.e.blocks.grow(self.table, n_tokens)

    def release(self):
        if self.table:
            self.e.blocks.release(self.table)
        self.table = []

    def forward(self, toks: list[int], all_logits: bool) -> torch.Tensor:
        """Run `toks` at positions len..len+n-1; returns logits [n, V] (or [1, V])."""
        e = self.e
        n = len(toks)
        self.ensure(self.len + n)
        bs = e.ecfg.block_size
        pos = list(range(self.len, self.len + n))
        slots = [self.table[p // bs] * bs + p % bs for p in pos]
        dev = e.device
        t = lambda a, dt: torch.tensor(a, dtype=dt, device=dev)  # noqa: E731
        last = list(range(n)) if all_logits else [n - 1]
        # every requested row is scored by presenting each position as its own "sequence" sharing
        # one block table: causal attention over the cache is identical either way
        if all_logits and n > 1:
            S = n
            bt = t([self.table] * S, torch.int32)
            q_start = t(list(range(S + 1)), torch.int32)
            seq_lens = t([self.len + i + 1 for i in range(n)], torch.int32)
            inp = StepInput(t(toks, torch.int32), t(pos, torch.int32), t(slots, torch.int64), bt, seq_lens,
                            t(list(range(n)), torch.int64), False, q_start=q_start, max_q=1)
        else:
            inp = StepInput(t(toks, torch.int32), t(pos, torch.int32), t(slots, torch.int64), t([self.table], torch.int32),
                            t([self.len + n], torch.int32), t(last, torch.int64), n == 1,
                            q_start=t([0, n], torch.int32), max_q=n)
        logits = e.runner.forward(inp).float()
        self.len += n
        return logits


def _probs(logits: torch.Tensor, p: SamplingParams) -> torch.Tensor:
    """Sampling distribution of every row of ``logits`` [R, V] (temperature, top-k, top-p, min-p in
    that order, as the host samplers apply them), computed on the logits' device for all rows at
    once.  Greedy: one-hot argmax."""
    if p.temperature <= 0:
        out = torch.zeros_like(logits)
        out.scatter_(-1, logits.argmax(-1, keepdim=True), 1.0)
        return out
    lg = logits.float() / p.temperature
    V = lg.shape[-1]
    if 0 < p.top_k < V:
        th = torch.topk(lg, p.top_k, dim=-1).values[:, -1:]
        lg = lg.masked_fill(lg < th, -float("inf"))
    if p.top_p < 1.0:
        sl, si = torch.sort(lg, dim=-1, descending=True)
        pr = torch.softmax(sl, -1)
        remove = (pr.cumsum(-1) - pr) >= p.top_p
        remove[:, 0] = False
        lg = lg.scatter(-1, si, sl.masked_fill(remove, -float("inf")))
    if p.min_p > 0.0:
        pr = torch.softmax(lg, -1)
        lg = lg.masked_fill(pr < p.min_p * pr.amax(-1, keepdim=True), -float("inf"))
    return torch.softmax(lg, -1)


def verify_drafts(ps: torch.Tensor, qs: torch.Tensor, drafts: torch.Tensor, greedy: bool,
                  gen: torch.Generator | None = None, seed: int | None = None, step: int = 0) -> tuple[int, list[int]]:
    """Rejection step of speculative decoding for k drafted tokens, on the device of ``ps``.

    ps: target distributions [k+1, V] (rows for the positions of d1..dk and the bonus position);
    qs: draft distributions [k, V]; drafts: int64 [k].  Returns (number accepted, tokens to append):
    the accepted prefix plus either the correction sampled from norm(max(0, p - q)) at the first
    rejection or the bonus token sampled from the last target row.  Greedy: accept while the
    target's argmax agrees, then append the target's argmax.  One host synchronization.

    On a GPU with ``seed`` given, the whole step is one kernel (K14, csrc/kernels/sampler.cu; its
    uniforms come from Philox keyed by ``seed`` at counter ``step``) and the result is one 4*(k+2)-byte
    read; otherwise the torch ops below (CPU engine, or a caller-supplied torch.Generator)."""
    k = drafts.numel()
    if ps.is_cuda and seed is not None:
        from ..ops import require_ext

        out = torch.empty(k + 2, dtype=torch.int32, device=ps.device)
        require_ext().spec_verify(ps.float().contiguous(), None if greedy else qs.float().contiguous(),
                                  drafts.to(torch.int64), int(greedy), int(seed) & ((1 << 63) - 1), int(step), out)
        res = out.tolist()
        n_acc = res[0]
        return n_acc, res[1:n_acc + 2]
    ar = torch.arange(k, device=ps.device)
    if greedy:
        tgt = ps.argmax(-1)  # [k+1]
        ok = tgt[:k] == drafts
    else:
        px = ps[ar, drafts]
        qx = qs[ar, drafts].clamp_min(1e-20)
        u = torch.rand(k, generator=gen, device=ps.device) if gen is not None else torch.rand(k, device=ps.device)
        ok = u < torch.clamp(px / qx, max=1.0)
    n_acc = int(torch.cumprod(ok.to(torch.int32), 0).sum()) if k else 0
    acc = drafts[:n_acc].tolist()
    if greedy:
        return n_acc, acc + [int(tgt[n_acc])]
    if n_acc < k:
        r = (ps[n_acc] - qs[n_acc]).clamp_min(0)
        tot = r.sum()
        r = r / tot if float(tot) > 0 else ps[n_acc]
    else:
        r = ps[k]
    return n_acc, acc + [int(torch.multinomial(r, 1, generator=gen))]


def lookup_drafts(tokens: list[int], k: int, n_max: int = 3, n_min: int = 1) -> list[int]:
    """Prompt-lookup drafting (no draft model): find the most recent earlier occurrence of the
    context's last n tokens (longest n first, n_max down to n_min) and propose the k tokens that
    followed it.  Pays off when the output repeats spans of its input (code edits, extraction,
    retrieval answers, summaries); returns [] when no n-gram recurs."""
    L = len(tokens)
    for n in range(min(n_max, L - 1), n_min - 1, -1):
        tail = tokens[L - n:]
        first = tail[0]
        for i in range(L - n - 1, -1, -1):
            if tokens[i] == first and tokens[i:i + n] == tail:
                cont = tokens[i + n:i + n + k]
                if cont:
                    return cont
    return []


class SpeculativeDecoder:
    """``draft`` is a draft engine (model drafting) or None: prompt-lookup drafting, whose drafts
    are deterministic (q is one-hot at the proposed token), so the rejection step accepts a
    drafted token x with probability p(x) and otherwise samples from p with x removed; the output
    distribution stays the target's either way."""

    def __init__(self, target, draft, cfg: SpeculativeConfig | None = None, lookup_ngram: int = 3):
        self.t = target
        self.d = draft
        self.cfg = cfg or SpeculativeConfig()
        self.lookup_ngram = lookup_ngram
        if draft is not None and target.cfg.vocab != draft.cfg.vocab:
            raise ValueError("draft and target must share a vocabulary")
        self.stats = SpecStats()
        target.spec_stats = self.stats

    @torch.no_grad()
    def generate(self, prompt: list[int], params: SamplingParams) -> SpecResult:
        t0 = time.perf_counter()
        dev = self.t.device
        gen = torch.Generator(device=dev).manual_seed(params.seed or 1234)
        greedy = params.temperature <= 0
        ts, ds = _Seq(self.t), (_Seq(self.d) if self.d is not None else None)
        try:
            # invariant: the target cache holds every token but the last; the draft may lag behind
            tokens = list(prompt)
            if len(prompt) > 1:
                ts.forward(prompt[:-1], False)
            out: list[int] = []
            k = self.cfg.draft_max
            reason = "length"
            while len(out) < params.max_tokens:
                k = max(self.cfg.draft_min, min(k, params.max_tokens - len(out)))
                last = tokens[-1]
                # 1) draft up to k tokens: autoregressively with the draft model (its first call
                # catches its cache up), or by prompt lookup
                drafts, qs = [], []
                if ds is not None:
                    feed = tokens[ds.len:]
                    for _ in range(k):
                        q = _probs(ds.forward(feed, False)[-1:], params)  # [1, V] on the device
                        cur = int(q.argmax()) if greedy else int(torch.multinomial(q[0], 1, generator=gen))
                        drafts.append(cur)
                        qs.append(q)
                        feed = [cur]
                else:
                    drafts = lookup_drafts(tokens, k, self.lookup_ngram)
                k_used = len(drafts)
                # 2) target scores [last, d1..dk] in one forward -> k+1 distributions
                ps = _probs(ts.forward([last] + drafts, True), params)
                if ds is None:
                    q1 = torch.zeros(k_used, ps.shape[-1], device=ps.device)
                    if k_used:
                        q1[torch.arange(k_used, device=ps.device), torch.tensor(drafts, device=ps.device)] = 1.0
                    qs = [q1]
                # 3) accept / reject on the device (one host synchronization); with nothing drafted
                # (no recurring n-gram) this is a plain decode step
                if k_used:
                    n_acc, new = verify_drafts(ps, torch.cat(qs), torch.tensor(drafts, dtype=torch.int64,
                                                                                device=ps.device),
                                               greedy, gen, seed=params.seed or 1234, step=len(out))
                else:
                    n_acc = 0
                    new = [int(ps[0].argmax()) if greedy else int(torch.multinomial(ps[0], 1, generator=gen))]
                if k_used and n_acc == k_used:
                    self.stats.bonus += 1
                self.stats.drafted += k_used
                self.stats.accepted += n_acc
                self.stats.steps += 1
                # 4) roll the caches back to the accepted prefix
                n_old = len(tokens)
                ts.len = n_old + n_acc
                if ds is not None:
                    ds.len = min(ds.len, n_old + n_acc)
                stop = False
                for tok in new:
                    out.append(tok)
                    tokens.append(tok)
                    if (not params.ignore_eos and tok in self.t.cfg.eos_ids) or tok in params.stop_token_ids:
                        reason, stop = "stop", True
                        break
                    if len(out) >= params.max_tokens:
                        stop = True
                        break
                if stop:
                    break
                if self.cfg.adaptive and k_used:
                    if n_acc == k_used:
                        k += 1
                    elif n_acc == 0:
                        k -= 1
                    k = max(self.cfg.draft_min, min(k, self.cfg.draft_max))
            return SpecResult(out, self.stats.acceptance_rate, self.stats, time.perf_counter() - t0, reason)
        finally:
            ts.release()
            if ds is not None:
                ds.release()
