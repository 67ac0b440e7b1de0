"""Request / sequence state tracked by the scheduler.

Parity: ``ActiveSequence`` (``advanced/src/continuous_batching.rs:16``) and ``BatchRequest``
(``advanced/src/batch_engine.rs:28``).
"""
from __future__ import annotations

import enum
import itertools
import time
from dataclasses import dataclass, field
from typing import Any, Callable

from .sampling_params import SamplingParams

_ids = itertools.count()


class SeqStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"


@dataclass(eq=False)  # identity semantics: membership tests in scheduler lists stay O(1) per item
class Sequence:
    prompt: list[int]
    params: SamplingParams
    request_id: str = ""
    seq_id: int = field(default_factory=lambda: next(_ids))
    output: list[int] = field(default_factory=list)
    logprobs: list[float] = field(default_factory=list)
    top_logprobs: list[list[tuple[int, float]]] = field(default_factory=list)
    block_table: list[int] = field(default_factory=list)
    n_cached: int = 0           # tokens whose K/V are in the cache
    status: SeqStatus = SeqStatus.WAITING
    finish_reason: str | None = None
    arrival: float = field(default_factory=time.perf_counter)
    first_token_time: float | None = None
    finish_time: float | None = None
    n_preempted: int = 0
    prefix_hit: int = 0
    on_token: Callable[["Sequence", int], None] | None = None
    grammar_state: Any = None
    host_sampler: Any = None
    # (first position, f32 [n, hidden] device tensor): prompt positions whose input embedding is
    # given instead of the token's (multimodal prompts); such prompts bypass the prefix cache
    embeds: Any = None
    window_freed: int = 0  # leading block-table entries released by the sliding window
    # bumped whenever block_table is replaced or rewritten (not when it only grows), so that packed
    # decode inputs can re-send only the entries appended since the previous step
    bt_gen: int = 0

    @property
    def tokens(self) -> list[int]:
        return self.prompt + self.output

    @property
    def last_token(self) -> int:
        return self.output[-1] if self.output else self.prompt[-1]

    def last_tokens(self, n: int) -> list[int]:
        """The last ``n`` tokens (prompt + output) without building the whole list."""
        if n <= len(self.output):
            return self.output[len(self.output) - n:]
        k = n - len(self.output)
        return self.prompt[max(0, len(self.prompt) - k):] + self.output

    @property
    def n_tokens(self) -> int:
        return len(self.prompt) + len(self.output)

    @property
    def n_uncached(self) -> int:
        return self.n_tokens - self.n_cached

    @property
    def is_prefill(self) -> bool:
        return self.n_uncached > 1 or not self.output and self.n_cached < len(self.prompt)

    @property
    def finished(self) -> bool:
        return self.status == SeqStatus.FINISHED

    @property
    def ttft(self) -> float | None:
        return None if self.first_token_time is None else self.first_token_time - self.arrival
