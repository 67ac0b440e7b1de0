"""High-level text API: load a GGUF model, generate / stream / chat with strings, batch prompts.

Parity: the ``barq_inference::client::{Client, GenerationConfig}`` API that the reference's examples
program against (``examples/basic_inference.rs``, ``examples/advanced_inference.rs``,
``examples/simple_inference.rs``) but that no crate of the reference defines.  Here it is a thin
layer over the engine (CUDA engine on a GPU, CPU engine otherwise), the GGUF tokenizer and the chat
template of the model.

    from barq_inference_b200.client import Client, GenerationConfig
    c = Client.from_gguf("model.gguf")
    print(c.generate("Hello", GenerationConfig(max_tokens=32, temperature=0)).text)
    for piece in c.stream("Tell me a story"):
        print(piece, end="")
    c.chat([{"role": "user", "content": "Give me JSON"}], GenerationConfig(json_mode=True))
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Iterator

from .engine.sampling_params import SamplingParams


@dataclass
class GenerationConfig:
    max_tokens: int = 128
    temperature: float = 0.8
    top_k: int = 40
    top_p: float = 0.95
    min_p: float = 0.0
    repetition_penalty: float = 1.0
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    seed: int = 0
    json_mode: bool = False
    json_schema: dict | None = None
    grammar: str | None = None  # GBNF
    stop: list[str] = field(default_factory=list)

    def sampling(self) -> SamplingParams:
        return SamplingParams(max_tokens=self.max_tokens, temperature=self.temperature, top_k=self.top_k,
                              top_p=self.top_p, min_p=self.min_p, repetition_penalty=self.repetition_penalty,
                              frequency_penalty=self.frequency_penalty, presence_penalty=self.presence_penalty,
                              seed=self.seed, json_mode=self.json_mode or self.json_schema is not None,
                              json_schema=self.json_schema, grammar=self.grammar)


@dataclass
class Response:
    text: str
    tokens: list[int]
    finish_reason: str
    prompt_tokens: int
    ttft_s: float | None
    latency_s: float

    @property
    def tokens_per_second(self) -> float:
        return len(self.tokens) / self.latency_s if self.latency_s > 0 else 0.0


def _cut_at_stop(text: str, stops: list[str]) -> tuple[str, bool]:
    hits = [i for i in (text.find(s) for s in stops if s) if i >= 0]
    return (text[: min(hits)], True) if hits else (text, False)


class Client:
    def __init__(self, engine, tokenizer, chat_template=None):
        self.engine = engine
        self.tok = tokenizer
        if chat_template is None:
            from .tokenizer import ChatTemplate

            chat_template = ChatTemplate("generic")
        self.template = chat_template

    @staticmethod
    def from_gguf(path: str, device: str | None = None, **engine_kw) -> "Client":
        """Loads ``path`` (split files too) onto ``device`` (``cuda`` when a GPU is visible, else
        ``cpu``); ``engine_kw`` go to ``EngineConfig`` (GPU engine)."""
        import torch

        from .gguf import read_gguf_split
        from .models.config import attach_rope_factors, config_from_gguf
        from .models.weights import tensors_from_gguf
        from .tokenizer import ChatTemplate, GGUFTokenizer, synthetic_tokenizer

        g = read_gguf_split(path)
        cfg = attach_rope_factors(config_from_gguf(g.metadata, set(g.tensors)), g)
        try:
            tok = GGUFTokenizer.from_metadata(g.metadata)
        except ValueError:
            tok = synthetic_tokenizer(cfg.vocab)
        tmpl = ChatTemplate.for_arch(cfg.arch, g.metadata)
        device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        tensors = tensors_from_gguf(g, device="cpu")
        if device == "cpu":
            from .engine.cpu_engine import CPUEngine

            eng = CPUEngine(cfg, tensors, max_model_len=int(engine_kw.get("max_model_len", cfg.max_ctx)))
        else:
            from .engine.engine import Engine, EngineConfig

            kw = {"max_model_len": cfg.max_ctx, **engine_kw, "device": device}
            eng = Engine(cfg, tensors, EngineConfig(**kw))
        eng.tokenizer = tok
        return Client(eng, tok, tmpl)

    # ------------------------------------------------------------------ prompts
    def encode(self, text: str) -> list[int]:
        return self.tok.encode(text)

    def chat_prompt(self, messages: list[dict]) -> list[int]:
        text = self.template.render(messages, add_generation_prompt=True)
        return self.tok.encode(text, add_special=not text.startswith(getattr(self.template, "bos_token", "") or "\0"))

    # ------------------------------------------------------------------ generation
    def _run(self, ids: list[int], cfg: GenerationConfig) -> Iterator[tuple[str, int | None, object]]:
        """Yields (text delta, token, sequence) as tokens are sampled; the last item has token None."""
        from .tokenizer import StreamDecoder

        dec = StreamDecoder(self.tok)
        pending: list[int] = []
        seq = self.engine.add_request(ids, cfg.sampling(), on_token=lambda s, t: pending.append(t))
        eos = set(self.engine.cfg.eos_ids)
        while True:
            while not pending and self.engine.has_work():
                self.engine.step()
            if not pending:
                break
            t = pending.pop(0)
            if t < 0:
                break
            if t in eos and not seq.params.ignore_eos:
                continue
            yield dec.push(t), t, seq
        yield dec.flush(), None, seq

    def stream(self, prompt: str | list[int], config: GenerationConfig | None = None) -> Iterator[str]:
        """Text pieces as they are generated (stop strings end the stream)."""
        cfg = config or GenerationConfig()
        ids = self.encode(prompt) if isinstance(prompt, str) else list(prompt)
        text = ""
        for piece, _, _ in self._run(ids, cfg):
            if not piece:
                continue
            if cfg.stop:
                cut, hit = _cut_at_stop(text + piece, cfg.stop)
                if hit:
                    if len(cut) > len(text):
                        yield cut[len(text):]
                    return
            text += piece
            yield piece

    def generate(self, prompt: str | list[int], config: GenerationConfig | None = None) -> Response:
        cfg = config or GenerationConfig()
        ids = self.encode(prompt) if isinstance(prompt, str) else list(prompt)
        t0 = time.perf_counter()
        ttft = None
        text, toks, seq = "", [], None
        for piece, t, seq in self._run(ids, cfg):
            if t is not None:
                toks.append(t)
                if ttft is None:
                    ttft = time.perf_counter() - t0
            text += piece
        reason = (seq.finish_reason if seq is not None else None) or "stop"
        if cfg.stop:
            text, hit = _cut_at_stop(text, cfg.stop)
            reason = "stop" if hit else reason
        return Response(text, toks, reason, len(ids), ttft, time.perf_counter() - t0)

    def generate_batch(self, prompts: list[str], config: GenerationConfig | None = None) -> list[Response]:
        """All prompts in one continuously batched run."""
        from .tokenizer import StreamDecoder

        cfg = config or GenerationConfig()
        t0 = time.perf_counter()
        ids = [self.encode(p) for p in prompts]
        res = self.engine.generate(ids, cfg.sampling())
        out = []
        eos = set(self.engine.cfg.eos_ids)
        for p, r in zip(ids, res):
            dec = StreamDecoder(self.tok)  # same text as streaming (keeps a leading space)
            text = "".join(dec.push(t) for t in r.tokens if t not in eos) + dec.flush()
            reason = r.finish_reason or "stop"
            if cfg.stop:
                text, hit = _cut_at_stop(text, cfg.stop)
                reason = "stop" if hit else reason
            out.append(Response(text, r.tokens, reason, len(p), r.ttft_s, time.perf_counter() - t0))
        return out

    def chat(self, messages: list[dict], config: GenerationConfig | None = None) -> Response:
        return self.generate(self.chat_prompt(messages), config)
