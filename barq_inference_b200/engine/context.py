"""Low-level single-sequence API: feed tokens, get logits, sample, roll back.

Parity: ``ModelContext::{encode, decode, sample}`` and ``Batch::from_tokens``
(``models/src/context.rs:391-556``), the API the reference's user guide programs against.  Here a
context is one sequence's attention state inside an engine:

* CUDA engine: pages borrowed from the engine's KV pool, driven straight through its model runner
  (the same path speculative decoding uses), so the state lives on the device; ``close`` returns
  the pages.
* CPU engine: the fp32 reference forward with a per-context K/V cache.

    ctx = ModelContext(engine)
    logits = ctx.encode([1, 2, 3, 4])          # [1, vocab]: logits after the last token
    tok = ctx.sample(logits, temperature=0.8, top_k=40, top_p=0.95)
    logits = ctx.decode(tok)
    ctx.truncate(2)                            # forget everything after the first 2 tokens
"""
from __future__ import annotations

import torch

from .sampling_params import SamplingParams


class ModelContext:
    def __init__(self, engine, seed: int = 0):
        self.engine = engine
        self.tokens: list[int] = []
        self._gen = torch.Generator().manual_seed(seed or 1234)
        if hasattr(engine, "sched"):  # CUDA engine: paged state through the runner
            from .speculative import _Seq

            self._seq = _Seq(engine)
            self._cache = None
        else:  # CPU engine: reference forward with its own cache
            self._seq = None
            self._cache: dict | None = {}

    @property
    def n_past(self) -> int:
        return len(self.tokens)

    def encode(self, tokens: list[int], all_logits: bool = False) -> torch.Tensor:
        """Append ``tokens``; returns fp32 logits [n, vocab] (``all_logits``) or [1, vocab] for the last."""
        tokens = [int(t) for t in tokens]
        if not tokens:
            raise ValueError("encode: no tokens")
        vocab = self.engine.cfg.vocab
        if any(t < 0 or t >= vocab for t in tokens):
            raise ValueError("encode: token id out of range")
        limit = getattr(getattr(self.engine, "ecfg", None), "max_model_len", None) or getattr(
            self.engine, "max_model_len", None)
        if limit is not None and self.n_past + len(tokens) > limit:
            raise ValueError(f"encode: context of {self.n_past + len(tokens)} tokens exceeds {limit}")
        if self._seq is not None:
            lg = self._seq.forward(tokens, all_logits)
        else:
            with torch.no_grad():
                lg = self.engine.model.forward(tokens, self._cache)
            lg = lg if all_logits else lg[-1:]
        self.tokens += tokens
        return lg.float().cpu()

    def decode(self, token: int) -> torch.Tensor:
        """One token in, logits [1, vocab] out."""
        return self.encode([token])

    def sample(self, logits: torch.Tensor, temperature: float = 0.8, top_k: int = 40, top_p: float = 0.95,
               min_p: float = 0.0, repetition_penalty: float = 1.0) -> int:
        from ..sampling.host_samplers import sample_chain

        p = SamplingParams(temperature=temperature, top_k=top_k, top_p=top_p, min_p=min_p,
                           repetition_penalty=repetition_penalty)
        return sample_chain(logits.reshape(-1), p, self.tokens, self._gen)

    def truncate(self, n: int) -> None:
        """Keep the first ``n`` tokens' state (roll back speculative or rejected continuations)."""
        if n < 0 or n > self.n_past:
            raise ValueError(f"truncate to {n}: context holds {self.n_past} tokens")
        if self._seq is not None:
            self._seq.len = n
        else:
            for k, v in list(self._cache.items()):
                if isinstance(k, tuple):
                    self._cache[k] = v[:n]
            self._cache["pos"] = n
        self.tokens = self.tokens[:n]

    def reset(self) -> None:
        self.truncate(0)

    def close(self) -> None:
        if self._seq is not None:
            self._seq.release()
        self.tokens = []

    def __enter__(self) -> "ModelContext":
        return self

    def __exit__(self, *exc) -> None:
        self.close()
