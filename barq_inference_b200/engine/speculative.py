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
from dataclasses import dataclass, field

import numpy as np
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
    if p.temperature <= 0:
        out = torch.zeros_like(logits)
        out.scatter_(-1, logits.argmax(-1, keepdim=True), 1.0)
        return out
    from ..sampling.host_samplers import min_p_filter, top_k_filter, top_p_filter

    rows = []
    for lg in logits:
        lg = top_k_filter(lg / p.temperature, p.top_k)
        lg = top_p_filter(lg, p.top_p)
        lg = min_p_filter(lg, p.min_p)
        rows.append(torch.softmax(lg, -1))
    return torch.stack(rows)


class SpeculativeDecoder:
    def __init__(self, target, draft, cfg: SpeculativeConfig | None = None):
        self.t = target
        self.d = draft
        self.cfg = cfg or SpeculativeConfig()
        if target.cfg.vocab != draft.cfg.vocab:
            raise ValueError("draft and target must share a vocabulary")
        self.stats = SpecStats()
        target.spec_stats = self.stats

    @torch.no_grad()
    def generate(self, prompt: list[int], params: SamplingParams) -> SpecResult:
        t0 = time.perf_counter()
        gen = torch.Generator(device="cpu").manual_seed(params.seed or 1234)
        ts, ds = _Seq(self.t), _Seq(self.d)
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
                # 1) draft k tokens autoregressively (first call catches the draft cache up)
                drafts, qs = [], []
                feed = tokens[ds.len:]
                for _ in range(k):
                    ql = ds.forward(feed, False)[-1:]
                    q = _probs(ql.cpu(), params)[0]
                    cur = int(torch.argmax(q)) if params.temperature <= 0 else int(torch.multinomial(q, 1, generator=gen))
                    drafts.append(cur)
                    qs.append(q)
                    feed = [cur]
                # 2) target scores [last, d1..dk] in one forward -> k+1 distributions
                pl = ts.forward([last] + drafts, True).cpu()
                ps = _probs(pl, params)
                # 3) accept / reject
                n_acc = 0
                new = []
                for i, x in enumerate(drafts):
                    p, q = ps[i], qs[i]
                    if params.temperature <= 0:
                        ok = int(torch.argmax(p)) == x
                    else:
                        ok = torch.rand((), generator=gen).item() < min(1.0, float(p[x] / max(float(q[x]), 1e-20)))
                    if ok:
                        new.append(x)
                        n_acc += 1
                        continue
                    if params.temperature <= 0:
                        new.append(int(torch.argmax(p)))
                    else:
                        r = (p - q).clamp_min(0)
                        r = r / r.sum() if r.sum() > 0 else p
                        new.append(int(torch.multinomial(r, 1, generator=gen)))
                    break
                else:
                    p = ps[k]
                    bonus = int(torch.argmax(p)) if params.temperature <= 0 else int(torch.multinomial(p, 1, generator=gen))
                    new.append(bonus)
                    self.stats.bonus += 1
                self.stats.drafted += k
                self.stats.accepted += n_acc
                self.stats.steps += 1
                # 4) roll the caches back to the accepted prefix
                n_old = len(tokens)
                ts.len = n_old + n_acc
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
                if self.cfg.adaptive:
                    if n_acc == k:
                        k += 1
                    elif n_acc == 0:
                        k -= 1
                    k = max(self.cfg.draft_min, min(k, self.cfg.draft_max))
            return SpecResult(out, self.stats.acceptance_rate, self.stats, time.perf_counter() - t0, reason)
        finally:
            ts.release()
            ds.release()
