"""``RemoteClient``: the text-level ``Client`` API (``generate`` / ``stream`` / ``chat`` /
``generate_batch``) against a running OpenAI-compatible server (``barq-http`` or ``barq
http-server``) instead of an in-process engine, so application code moves from one process to a
served deployment by changing the constructor.

Standard library only (``http.client``); streaming reads the server's SSE chunks as they arrive.
Token ids are not returned by the HTTP API, so ``Response.tokens`` is empty and ``completion``
counts come from the server's ``usage``.
"""
from __future__ import annotations

import http.client
import json
import time
from dataclasses import dataclass
from typing import Iterator
from urllib.parse import urlparse

from .client import GenerationConfig, Response


@dataclass
class RemoteResponse(Response):
    completion_tokens: int = 0


class RemoteClient:
    def __init__(self, url: str = "http://127.0.0.1:8000", api_key: str | None = None, model: str = "barq",
                 timeout: float = 600.0):
        u = urlparse(url)
        if u.scheme not in ("http", ""):
            raise ValueError("RemoteClient speaks plain HTTP (put TLS in front of the server)")
        self.host, self.port = u.hostname or "127.0.0.1", u.port or 80
        self.api_key, self.model, self.timeout = api_key, model, timeout

    # ------------------------------------------------------------------ plumbing
    def _body(self, cfg: GenerationConfig, stream: bool) -> dict:
        b = {"model": self.model, "max_tokens": cfg.max_tokens, "temperature": cfg.temperature, "top_k": cfg.top_k,
             "top_p": cfg.top_p, "min_p": cfg.min_p, "repetition_penalty": cfg.repetition_penalty,
             "frequency_penalty": cfg.frequency_penalty, "presence_penalty": cfg.presence_penalty,
             "seed": cfg.seed, "stream": stream}
        if stream:
            b["stream_options"] = {"include_usage": True}
        if cfg.stop:
            b["stop"] = list(cfg.stop)
        if cfg.json_schema is not None:
            b["response_format"] = {"type": "json_schema", "json_schema": {"schema": cfg.json_schema}}
        elif cfg.json_mode:
            b["response_format"] = {"type": "json_object"}
        if cfg.grammar:
            b["grammar"] = cfg.grammar
        return b

    def _post(self, path: str, body: dict):
        c = http.client.HTTPConnection(self.host, self.port, timeout=self.timeout)
        headers = {"Content-Type": "application/json"}
        if self.api_key:
            headers["Authorization"] = f"Bearer {self.api_key}"
        c.request("POST", path, body=json.dumps(body), headers=headers)
        r = c.getresponse()
        if r.status != 200:
            msg = r.read().decode(errors="replace")
            c.close()
            try:
                msg = json.loads(msg)["error"]["message"]
            except (ValueError, KeyError, TypeError):
                pass
            raise RuntimeError(f"HTTP {r.status}: {msg}")
        return c, r

    def _events(self, path: str, body: dict) -> Iterator[dict]:
        c, r = self._post(path, body)
        try:
            buf = b""
            while True:
                chunk = r.read1(65536) if hasattr(r, "read1") else r.read(65536)
                if not chunk:
                    return
                buf += chunk
                while b"\n\n" in buf:
                    ev, buf = buf.split(b"\n\n", 1)
                    if not ev.startswith(b"data: "):
                        continue
                    if ev[6:] == b"[DONE]":
                        return
                    yield json.loads(ev[6:])
        finally:
            c.close()

    @staticmethod
    def _piece(obj: dict) -> tuple[str, str | None]:
        ch = (obj.get("choices") or [{}])[0]
        text = ch.get("text") if "text" in ch else (ch.get("delta") or {}).get("content") or ""
        return text or "", ch.get("finish_reason")

    def _stream(self, path: str, body: dict):
        """Yields (text piece, finish reason | None, usage | None)."""
        for obj in self._events(path, body):
            if obj.get("usage"):
                yield "", None, obj["usage"]
                continue
            text, fin = self._piece(obj)
            yield text, fin, None

    # ------------------------------------------------------------------ Client API
    def stream(self, prompt: str | list[int], config: GenerationConfig | None = None) -> Iterator[str]:
        cfg = config or GenerationConfig()
        for text, _, _ in self._stream("/v1/completions", {**self._body(cfg, True), "prompt": prompt}):
            if text:
                yield text

    def _collect(self, path: str, body: dict) -> RemoteResponse:
        t0 = time.perf_counter()
        ttft, parts, reason, usage = None, [], "stop", {}
        for text, fin, u in self._stream(path, body):
            if text:
                parts.append(text)
                if ttft is None:
                    ttft = time.perf_counter() - t0
            if fin:
                reason = fin
            if u:
                usage = u
        return RemoteResponse("".join(parts), [], reason, int(usage.get("prompt_tokens", 0)), ttft,
                              time.perf_counter() - t0, int(usage.get("completion_tokens", 0)))

    def generate(self, prompt: str | list[int], config: GenerationConfig | None = None) -> RemoteResponse:
        cfg = config or GenerationConfig()
        return self._collect("/v1/completions", {**self._body(cfg, True), "prompt": prompt})

    def chat(self, messages: list[dict], config: GenerationConfig | None = None) -> RemoteResponse:
        cfg = config or GenerationConfig()
        return self._collect("/v1/chat/completions", {**self._body(cfg, True), "messages": messages})

    def generate_batch(self, prompts: list[str], config: GenerationConfig | None = None) -> list[RemoteResponse]:
        """All prompts in one request (the server batches them)."""
        cfg = config or GenerationConfig()
        t0 = time.perf_counter()
        c, r = self._post("/v1/completions", {**self._body(cfg, False), "prompt": list(prompts)})
        try:
            out = json.loads(r.read())
        finally:
            c.close()
        dt = time.perf_counter() - t0
        return [RemoteResponse(ch.get("text", ""), [], ch.get("finish_reason") or "stop", 0, None, dt)
                for ch in out["choices"]]
