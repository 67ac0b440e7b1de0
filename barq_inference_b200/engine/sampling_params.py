"""Per-request sampling parameters.

Parity: the reference's sampler chain configuration (``sampling/src/lib.rs:54-65``), the CLI
defaults (``cli/src/main.rs:77-116``: temperature 0.8, top-k 40, top-p 0.95) and the HTTP defaults
(``cli/src/server.rs``: max_tokens 128).
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class SamplingParams:
    max_tokens: int = 128
    temperature: float = 0.8
    top_k: int = 40
    top_p: float = 0.95
    min_p: float = 0.0
    typical_p: float = 1.0
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    penalty_last_n: int = 64
    mirostat: int = 0  # 0 off, 1 = v1, 2 = v2 (host-side sampler)
    mirostat_tau: float = 5.0
    mirostat_eta: float = 0.1
    xtc_probability: float = 0.0
    xtc_threshold: float = 0.1
    seed: int = 0
    stop_token_ids: list[int] = field(default_factory=list)
    ignore_eos: bool = False
    grammar: str | None = None  # GBNF text
    json_mode: bool = False
    json_schema: dict | None = None
    logprobs: bool = False     # record log p(token) of every sampled token (log-softmax of the raw logits)
    top_logprobs: int = 0      # ... and the most likely alternatives (0..20)

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0

    @property
    def needs_host_sampler(self) -> bool:
        return self.mirostat != 0 or self.typical_p < 1.0 or self.xtc_probability > 0.0

    @property
    def needs_penalties(self) -> bool:
        return self.repetition_penalty != 1.0 or self.frequency_penalty != 0.0 or self.presence_penalty != 0.0

    @staticmethod
    def greedy_params(max_tokens: int = 128, **kw) -> "SamplingParams":
        return SamplingParams(max_tokens=max_tokens, temperature=0.0, top_k=0, top_p=1.0, **kw)
