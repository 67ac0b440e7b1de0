"""CPU engine: the same request API as ``Engine`` on the fp32 reference forward.

Parity: the reference's only working path is the CPU f32 forward (``models/src/transformer.rs``,
``models/src/context.rs:391-556``).  This engine serves the same role here — ``--device cpu`` in the
CLI, the servers' tests, and the timed CPU baseline on the tiny config — while the CUDA engine is
the product.  It keeps one KV cache per sequence and decodes sequences round-robin, one token per
step each, with the host sampler chain and grammar masks.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from ..models.config import ModelConfig
from ..models.reference import ReferenceModel
from ..sampling.host_samplers import new_host_sampler, sample_chain
from .logprobs import record_logprobs
from .engine import GenerationResult
from .sampling_params import SamplingParams
from .sequence import Sequence, SeqStatus


class CPUEngine:
    def __init__(self, cfg: ModelConfig, tensors, max_model_len: int = 2048, ser_threshold: float = 0.0,
                 max_waiting: int = 0):
        self.cfg = cfg
        self.model = ReferenceModel(cfg, tensors, ser_threshold=ser_threshold)
        self.max_model_len = min(max_model_len, cfg.max_ctx)
        self.max_waiting = max_waiting  # admission control (0: no limit), as in the scheduler
        self.waiting: list[Sequence] = []
        self.running: list[Sequence] = []
        self.caches: dict[int, dict] = {}
        self.gens: dict[int, torch.Generator] = {}
        self.tokenizer = None
        self.step_count = 0
        self.timings = {"prefill_s": 0.0, "decode_s": 0.0, "prefill_tokens": 0, "decode_tokens": 0}
        # imported KV sessions (engine.session.import_session): (tokens, reference-forward cache)
        self.sessions: list[tuple[list[int], dict]] = []

    def add_request(self, prompt: list[int], params: SamplingParams | None = None, request_id: str = "",
                    on_token=None, embeds: tuple[int, torch.Tensor] | None = None) -> Sequence:
        params = params or SamplingParams()
        if not prompt:
            raise ValueError("empty prompt")
        if any(t < 0 or t >= self.cfg.vocab for t in prompt):
            raise ValueError("prompt token id out of range")
        if len(prompt) >= self.max_model_len:
            raise ValueError("prompt exceeds max_model_len")
        if self.max_waiting and len(self.waiting) >= self.max_waiting:
            from .scheduler import Overloaded

            raise Overloaded(f"{len(self.waiting)} requests already waiting; retry later")
        seq = Sequence(list(prompt), params, request_id=request_id, on_token=on_token)
        if embeds is not None:
            st, e = embeds
            if e.dim() != 2 or e.shape[1] != self.cfg.hidden or st < 0 or st + e.shape[0] > len(prompt):
                raise ValueError("embeds: need [n, hidden] rows inside the prompt")
            seq.embeds = (int(st), e.float().cpu())
        if params.grammar or params.json_mode or params.json_schema:
            from ..sampling.grammar_engine import make_grammar_state

            seq.grammar_state = make_grammar_state(self, params)
        if params.needs_host_sampler:
            seq.host_sampler = new_host_sampler(params, self.cfg.vocab)
        self.waiting.append(seq)
        return seq

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def abort(self, seq: Sequence) -> bool:
        """Stop generating for ``seq`` (e.g. its client disconnected)."""
        seq.on_token = None
        if seq in self.waiting:
            self.waiting.remove(seq)
        elif seq not in self.running:
            return False
        self._finish(seq, "abort")
        return True

    def embed(self, prompts: list[list[int]], normalize: bool = True) -> torch.Tensor:
        """Mean-pooled final-norm hidden states of each prompt ([N, hidden], fp32)."""
        from .embeddings import embed_cpu

        return embed_cpu(self, prompts, normalize)

    def _finish(self, s: Sequence, reason: str) -> None:
        s.status = SeqStatus.FINISHED
        s.finish_reason = reason
        s.finish_time = time.perf_counter()
        self.caches.pop(s.seq_id, None)
        if s in self.running:
            self.running.remove(s)

    @torch.no_grad()
    def step(self) -> list[Sequence]:
        while self.waiting:
            s = self.waiting.pop(0)
            s.status = SeqStatus.RUNNING
            self.running.append(s)
            self.caches[s.seq_id] = {}
            self.gens[s.seq_id] = torch.Generator().manual_seed(s.params.seed or s.seq_id)
            s.pending_prefill = True
        done = []
        for s in list(self.running):
            t0 = time.perf_counter()
            cache = self.caches[s.seq_id]
            if getattr(s, "pending_prefill", False):
                start = self._resume(s, cache)
                logits = self.model.forward(s.tokens[start:], cache, embeds=s.embeds)[-1]
                s.pending_prefill = False
                key = "prefill"
                n = s.n_tokens - start
            else:
                logits = self.model.forward([s.tokens[-1]], cache)[-1]
                key = "decode"
                n = 1
            s.n_cached = s.n_tokens
            raw = logits
            if s.grammar_state is not None:
                m = s.grammar_state.allowed_mask((self.cfg.vocab + 31) // 32)
                bits = np.unpackbits(m.view(np.uint8), bitorder="little")[: self.cfg.vocab].astype(bool)
                logits = logits.masked_fill(~torch.from_numpy(bits), float("-inf"))
            if s.host_sampler is not None:
                tok = s.host_sampler.sample(logits, s)
            else:
                tok = sample_chain(logits, s.params, s.tokens, self.gens[s.seq_id])
            if s.params.logprobs:
                record_logprobs(raw[None], [0], [tok], [s])
            self.timings[key + "_s"] += time.perf_counter() - t0
            self.timings[key + "_tokens"] += n
            if s.first_token_time is None:
                s.first_token_time = time.perf_counter()
            s.output.append(tok)
            if s.grammar_state is not None:
                s.grammar_state.accept(tok)
            if s.on_token is not None:
                s.on_token(s, tok)
            reason = None
            if not s.params.ignore_eos and tok in self.cfg.eos_ids:
                reason = "stop"
            elif tok in s.params.stop_token_ids:
                reason = "stop"
            elif s.grammar_state is not None and s.grammar_state.done():
                reason = "stop"
            elif len(s.output) >= s.params.max_tokens or s.n_tokens >= self.max_model_len:
                reason = "length"
            if reason:
                self._finish(s, reason)
                done.append(s)
                if s.on_token is not None:
                    s.on_token(s, -1)
        self.step_count += 1
        return done

    def _resume(self, s: Sequence, cache: dict) -> int:
        """Seeds ``cache`` from the longest imported session that is a strict prefix of the prompt;
        returns the number of positions that need no prefill."""
        if s.embeds is not None or not self.sessions:
            return 0
        toks = s.tokens
        best_k, best_c = 0, None
        for st, c in self.sessions:
            # usable length: the whole session if it is a strict prefix of the prompt, else the prompt
            # minus its last token when the session covers that (the last position must run for logits)
            if len(st) < len(toks) and toks[: len(st)] == st:
                k = len(st)
            elif len(st) >= len(toks) - 1 and st[: len(toks) - 1] == toks[:-1]:
                k = len(toks) - 1
            else:
                continue
            if k > best_k:
                best_k, best_c = k, c
        if best_c is None:
            return 0
        for key, t in best_c.items():  # the forward concatenates new rows into fresh tensors
            cache[key] = t[:best_k] if isinstance(key, tuple) else best_k
        return best_k

    def generate(self, prompts: list[list[int]], params=None) -> list[GenerationResult]:
        if params is None or isinstance(params, SamplingParams):
            params = [params or SamplingParams()] * len(prompts)
        seqs = [self.add_request(p, sp) for p, sp in zip(prompts, params)]
        while self.has_work():
            self.step()
        return [self._result(s) for s in seqs]

    def _result(self, s: Sequence) -> GenerationResult:
        return GenerationResult(s.prompt, s.output, s.finish_reason or "", s.ttft,
                                (s.finish_time or time.perf_counter()) - s.arrival, s.logprobs,
                                s.top_logprobs)
