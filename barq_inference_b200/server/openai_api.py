"""OpenAI-compatible HTTP API with true token-by-token SSE streaming.

Parity: ``cli/src/server.rs`` — routes ``GET /``, ``GET /v1/models``, ``POST /v1/completions``,
``POST /v1/chat/completions``, ``POST /v1/responses``, ``OPTIONS *`` (CORS), per-IP token-bucket rate
limiting (429 ``rate_limit_error``), request defaults (max_tokens 128, temperature 0.8, top_k 40,
top_p 0.95), ``/v1/responses`` accepting ``input`` / ``prompt`` / ``messages`` and
``max_output_tokens``, ids ``cmpl-`` / ``chatcmpl-`` / ``resp-<unix ts>``, SSE chunk objects
``text_completion.chunk``, ``chat.completion.chunk`` (role delta first) and ``response.chunk``,
``data: [DONE]``.  Added: ``/health``, ``/metrics`` (Prometheus), ``response_format`` JSON mode /
JSON schema, ``grammar`` (GBNF), ``tools`` / ``tool_choice`` (function calls constrained by the
tools' parameter schemas), ``stop``, ``seed``, ``n`` choices, ``stream_options.include_usage``,
per-request log lines with ``x-request-id``, 503 from admission control, and continuous batching
across concurrent requests.
"""
from __future__ import annotations

import asyncio
import dataclasses
import hmac
import json
import threading
import time
import uuid
from collections import OrderedDict
from typing import Any

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, PlainTextResponse, Response, StreamingResponse

from ..engine.sampling_params import SamplingParams
from ..engine.scheduler import Overloaded
from ..tokenizer import ChatTemplate, StreamDecoder
from ..utils.logging import request_logger
from .async_engine import AsyncEngine
from .metrics import InferenceMetrics, context_health
from .chat_tools import normalize_messages, tool_call_of, tool_names, tool_setup
from .request_params import DEFAULTS, sampling_params_from_request as _params  # noqa: F401

CORS = {"Access-Control-Allow-Origin": "*", "Access-Control-Allow-Methods": "GET, POST, OPTIONS",
        "Access-Control-Allow-Headers": "*"}


def _held_suffix(text: str, stops: list[str]) -> int:
    """Length of the longest end of ``text`` that is a proper prefix of a stop string."""
    hold = 0
    for x in stops:
        for n in range(min(len(x) - 1, len(text)), hold, -1):
            if text.endswith(x[:n]):
                hold = n
                break
    return hold


class RateLimiter:
    """Token bucket per client key; capacity = requests per minute, refilled continuously."""

    def __init__(self, rpm: int):
        self.capacity = float(max(1, rpm))
        self.refill = self.capacity / 60.0
        self.state: dict[str, tuple[float, float]] = {}
        self.lock = threading.Lock()

    def allow(self, key: str, now: float | None = None) -> bool:
        now = time.monotonic() if now is None else now
        with self.lock:
            tokens, last = self.state.get(key, (self.capacity, now))
            tokens = min(self.capacity, tokens + (now - last) * self.refill)
            ok = tokens >= 1.0
            self.state[key] = (tokens - 1.0 if ok else tokens, now)
            return ok


def _err(status: int, msg: str, kind: str = "invalid_request_error") -> JSONResponse:
    return JSONResponse({"error": {"message": msg, "type": kind}}, status_code=status, headers=CORS)


def _tool_calls(out: dict, body: dict) -> None:
    """Turn chat choices whose text is a function-call object into OpenAI ``tool_calls``."""
    names = tool_names(body)
    for i, ch in enumerate(out.get("choices", [])):
        call = tool_call_of((ch.get("message") or {}).get("content") or "", names)
        if call is not None:
            ch["message"] = {"role": "assistant", "content": None,
                             "tool_calls": [{"id": f"call_{out['id']}_{i}", "type": "function",
                                             "function": {"name": call["name"],
                                                          "arguments": json.dumps(call["arguments"])}}]}
            ch["finish_reason"] = "tool_calls"


class OpenAIServer:
    def __init__(self, engine, tokenizer, model_id: str = "barq", chat_template: ChatTemplate | None = None,
                 rate_limit_rpm: int = 0, arch: str = "llama", aengine=None, api_key: str | None = None):
        self.metrics = InferenceMetrics()
        # ``aengine``: a ready front with the AsyncEngine caller API (e.g. the data-parallel replica
        # router, whose ``engine`` argument is then itself)
        self.aengine = aengine if aengine is not None else AsyncEngine(engine, self.metrics)
        self.engine = engine
        self.tok = tokenizer
        self.model_id = model_id
        self.arch = arch
        self.template = chat_template or ChatTemplate("generic")
        self.limiter = RateLimiter(rate_limit_rpm) if rate_limit_rpm > 0 else None
        # optional shared secret: the /v1 routes need "Authorization: Bearer <key>" (401 otherwise)
        self.api_key = api_key or None
        self._tok_cache: OrderedDict[str, tuple[int, ...]] = OrderedDict()
        self._tok_lock = threading.Lock()
        self.tok_cache_size = 1024
        self.tok_cache_hits = 0
        self.app = self._build()

    # ------------------------------------------------------------------ helpers
    def _stops(self, body: dict) -> list[str]:
        s = body.get("stop")
        if s is None:
            return []
        return [s] if isinstance(s, str) else [str(x) for x in s]

    async def _run(self, prompt_ids: list[int], params: SamplingParams, stops: list[str]):
        """Yields (text_delta, finish_reason | None, logprob entries, tokens) per delta: the entries
        and the count of the generated tokens behind it; the finish comes last.  With stop strings,
        text that could still be the start of one is held back until it cannot, so no part of a stop
        string is ever sent."""
        dec = StreamDecoder(self.tok)
        text, sent, k, ntok = "", 0, 0, 0
        pend: list = []  # logprob entries of tokens whose text has not been yielded yet
        longest = max((len(x) for x in stops), default=0)
        async for item in self.aengine.stream(prompt_ids, params):
            if item.token is None:
                text += dec.flush()
                if len(text) > sent:
                    yield text[sent:], None, pend, ntok
                    pend, ntok = [], 0
                yield "", item.finish_reason or "stop", pend, ntok
                return
            idx, k = k, k + 1  # position of this token among the generated ones
            if item.token in self.engine.cfg.eos_ids and not params.ignore_eos:
                continue
            ntok += 1
            if params.logprobs:
                e = self._lp_entry(item, idx)
                if e is not None:
                    pend.append(e)
            before = len(text)
            text += dec.push(item.token)
            safe = len(text)
            if stops:
                hits = [text.find(x, max(0, before - longest)) for x in stops if x]
                hit = min((h for h in hits if h >= 0), default=-1)
                if hit >= 0:
                    yield text[sent:hit] if hit > sent else "", None, pend, ntok
                    yield "", "stop", [], 0
                    return
                safe -= _held_suffix(text, stops)
            if safe > sent:
                yield text[sent:safe], None, pend, ntok
                pend, ntok = [], 0
                sent = safe

    def _lp_entry(self, item, idx: int):
        """(token id, logprob, [(alt id, logprob), ...]) of the idx-th generated token, from the
        engine's per-sequence record (None when the engine did not record one)."""
        seq = item.seq
        lps = getattr(seq, "logprobs", None)
        if not lps or idx >= len(lps):
            return None
        tops = getattr(seq, "top_logprobs", None) or []
        return item.token, float(lps[idx]), list(tops[idx]) if idx < len(tops) else []

    def _lp_token(self, tid: int) -> tuple[str, list[int]]:
        b = self.tok.token_bytes(tid) if hasattr(self.tok, "token_bytes") else self.tok.decode([tid]).encode()
        return b.decode("utf-8", errors="replace"), list(b)

    def _lp_chat(self, entries: list) -> dict:
        """OpenAI chat form: {"content": [{token, logprob, bytes, top_logprobs: [...]}, ...]}."""
        out = []
        for tid, lp, top in entries:
            t, b = self._lp_token(tid)
            alts = []
            for aid, alp in top:
                at, ab = self._lp_token(aid)
                alts.append({"token": at, "logprob": alp, "bytes": ab})
            out.append({"token": t, "logprob": lp, "bytes": b, "top_logprobs": alts})
        return {"content": out}

    def _lp_text(self, entries: list, offset: int = 0) -> dict:
        """OpenAI completions form: tokens, token_logprobs, top_logprobs, text_offset."""
        toks, lps, tops, offs = [], [], [], []
        for tid, lp, top in entries:
            t, _ = self._lp_token(tid)
            toks.append(t)
            lps.append(lp)
            tops.append({self._lp_token(a)[0]: alp for a, alp in top} if top else None)
            offs.append(offset)
            offset += len(t)
        return {"tokens": toks, "token_logprobs": lps,
                "top_logprobs": tops if any(x is not None for x in tops) else None, "text_offset": offs}

    def _limit(self, request: Request) -> JSONResponse | None:
        if self.limiter is None:
            return None
        key = request.client.host if request.client else "unknown"
        if not self.limiter.allow(key):
            self.metrics.rate_limited += 1
            return _err(429, "rate limit exceeded; retry later", "rate_limit_error")
        return None

    async def _body(self, request: Request) -> dict:
        try:
            body = await request.json()
        except Exception:
            raise ValueError("request body is not valid JSON")
        if not isinstance(body, dict):
            raise ValueError("request body must be a JSON object")
        return body

    def _sse(self, gen):
        async def wrap():
            async for obj in gen:
                yield f"data: {json.dumps(obj)}\n\n"
            yield "data: [DONE]\n\n"

        return StreamingResponse(wrap(), media_type="text/event-stream",
                                 headers={**CORS, "Cache-Control": "no-cache"})

    async def _complete(self, prompt_ids, params, stops, kind: str, model: str, n_choices: int = 1):
        guard = self.metrics.begin()
        created = int(time.time())
        rid = {"text": "cmpl", "chat": "chatcmpl", "resp": "resp"}[kind] + f"-{created}{id(guard) % 100000}"

        # a batch of prompts (completions) gives n choices per prompt, indexed prompt-major
        batch = prompt_ids if prompt_ids and isinstance(prompt_ids[0], list) else [prompt_ids]

        async def one(b: int, i: int):
            # choice i samples with its own seed (a 0 seed already differs per request)
            p = dataclasses.replace(params, seed=params.seed + i) if (i and params.seed) else params
            parts, reason, n, lps = [], "stop", 0, []
            async for delta, fin, entries, ntok in self._run(batch[b], p, stops):
                if delta:
                    guard.first_token()
                    parts.append(delta)
                n += ntok
                lps += entries
                if fin:
                    reason = fin
            return "".join(parts), reason, n, lps

        try:
            outs = await asyncio.gather(*(one(b, i) for b in range(len(batch)) for i in range(n_choices)))
        except Exception:
            guard.fail()
            raise
        n_tok = sum(o[2] for o in outs)
        n_prompt = sum(len(x) for x in batch)
        guard.complete(n_prompt, n_tok)
        usage = {"prompt_tokens": n_prompt, "completion_tokens": n_tok, "total_tokens": n_prompt + n_tok}
        lp = params.logprobs
        if kind == "text":
            return {"id": rid, "object": "text_completion", "created": created, "model": model,
                    "choices": [{"index": i, "text": t, "finish_reason": r,
                                 "logprobs": self._lp_text(e) if lp else None}
                                for i, (t, r, _, e) in enumerate(outs)],
                    "usage": usage}
        if kind == "chat":
            return {"id": rid, "object": "chat.completion", "created": created, "model": model,
                    "choices": [{"index": i, "message": {"role": "assistant", "content": t}, "finish_reason": r,
                                 "logprobs": self._lp_chat(e) if lp else None}
                                for i, (t, r, _, e) in enumerate(outs)], "usage": usage}
        return {"id": rid, "object": "response", "created": created, "model": model, "output": outs[0][0],
                "usage": usage}

    async def _stream(self, prompt_ids, params, stops, kind: str, model: str, include_usage: bool = False):
        guard = self.metrics.begin()
        created = int(time.time())
        rid = {"text": "cmpl", "chat": "chatcmpl", "resp": "resp"}[kind] + f"-{created}{id(guard) % 100000}"
        n = 0
        try:
            if kind == "chat":
                yield {"id": rid, "object": "chat.completion.chunk", "created": created, "model": model,
                       "choices": [{"index": 0, "delta": {"role": "assistant"}, "finish_reason": None}]}
            offset = 0
            async for delta, fin, entries, ntok in self._run(prompt_ids, params, stops):
                if delta:
                    guard.first_token()
                n += ntok
                if not delta and not fin and not entries:
                    continue
                if kind == "text":
                    ch = {"index": 0, "text": delta, "finish_reason": fin}
                    if params.logprobs:
                        ch["logprobs"] = self._lp_text(entries, offset)
                    offset += len(delta)
                    yield {"id": rid, "object": "text_completion.chunk", "created": created, "model": model,
                           "choices": [ch]}
                elif kind == "chat":
                    ch = {"index": 0, "delta": ({"content": delta} if delta else {}), "finish_reason": fin}
                    if params.logprobs:
                        ch["logprobs"] = self._lp_chat(entries)
                    yield {"id": rid, "object": "chat.completion.chunk", "created": created, "model": model,
                           "choices": [ch]}
                else:
                    yield {"id": rid, "object": "response.chunk", "created": created, "model": model, "output": delta}
            guard.complete(len(prompt_ids), n)
            if include_usage:  # stream_options.include_usage: a final chunk with usage and no choices
                yield {"id": rid, "object": "chat.completion.chunk" if kind == "chat" else "text_completion.chunk",
                       "created": created, "model": model, "choices": [],
                       "usage": {"prompt_tokens": len(prompt_ids), "completion_tokens": n,
                                 "total_tokens": len(prompt_ids) + n}}
        finally:
            if not guard.done:
                guard.fail()

    def _encode(self, text: str) -> list[int]:
        """Tokenize with an LRU of recent prompts (repeated system prompts / retries skip the
        tokenizer; the role of the reference's prompt-processing cache, ``barq_core`` context)."""
        with self._tok_lock:
            hit = self._tok_cache.get(text)
            if hit is not None:
                self._tok_cache.move_to_end(text)
                self.tok_cache_hits += 1
                return list(hit)
        ids = self.tok.encode(text, add_special=True)
        if not ids:
            raise ValueError("empty prompt")
        with self._tok_lock:
            self._tok_cache[text] = tuple(ids)
            if len(self._tok_cache) > self.tok_cache_size:
                self._tok_cache.popitem(last=False)
        return ids

    def _chat_prompt(self, messages: Any) -> list[int]:
        text = self.template.render(normalize_messages(messages), add_generation_prompt=True)
        return self.tok.encode(text, add_special=not text.startswith(getattr(self.template, "bos_token", "") or "\0"))

    # ------------------------------------------------------------------ app
    def _build(self) -> FastAPI:
        app = FastAPI(title="barq-inference", docs_url=None, redoc_url=None)
        srv = self

        @app.middleware("http")
        async def cors(request: Request, call_next):
            if request.method == "OPTIONS":
                return Response(status_code=204, headers=CORS)
            if srv.api_key and request.url.path.startswith("/v1/") and not hmac.compare_digest(
                    request.headers.get("authorization", ""), f"Bearer {srv.api_key}"):
                return _err(401, "missing or invalid API key", "authentication_error")
            resp = await call_next(request)
            for k, v in CORS.items():
                resp.headers.setdefault(k, v)
            return resp

        @app.get("/")
        async def root():
            return {"object": "server.info", "model": srv.model_id, "architecture": srv.arch,
                    "endpoints": ["/v1/models", "/v1/responses", "/v1/completions", "/v1/chat/completions",
                                  "/v1/embeddings", "/tokenize", "/detokenize",
                                  "/health", "/metrics"]}

        @app.get("/v1/models")
        async def models():
            return {"object": "list", "data": [{"id": srv.model_id, "object": "model", "created": int(time.time()),
                                                "owned_by": "barq"}]}

        @app.get("/v1/models/{model_id:path}")
        async def model_info(model_id: str):
            if model_id != srv.model_id:
                return _err(404, f"model {model_id!r} not found", "not_found_error")
            return {"id": srv.model_id, "object": "model", "created": int(time.time()), "owned_by": "barq"}

        @app.get("/health")
        async def health():
            blocks = getattr(srv.engine, "blocks", None)
            used = blocks.n_used / blocks.num_blocks if blocks is not None else 0.0
            ok = srv.aengine.healthy
            body = {"status": "ok" if ok else "degraded", "kv_usage": used,
                    "context_health": context_health(used).value, "last_error": srv.aengine.last_error}
            return JSONResponse(body, status_code=200 if ok else 503)

        @app.get("/metrics")
        async def metrics():
            return PlainTextResponse(srv.metrics.prometheus(srv.engine), media_type="text/plain; version=0.0.4")

        async def handle(request: Request, kind: str):
            rid = request.headers.get("x-request-id") or uuid.uuid4().hex[:16]
            rlog = request_logger(rid)
            t0 = time.perf_counter()
            resp = await _handle(request, kind)
            ctx = {"endpoint": request.url.path, "status": resp.status_code,
                   "latency_ms": round((time.perf_counter() - t0) * 1000, 3),
                   "stream": isinstance(resp, StreamingResponse)}
            rlog.info("request %s", "accepted" if ctx["stream"] else "completed", extra={"context": ctx})
            resp.headers["x-request-id"] = rid
            return resp

        async def _handle(request: Request, kind: str):
            lim = srv._limit(request)
            if lim is not None:
                return lim
            try:
                body = await srv._body(request)
                model = body.get("model") or srv.model_id
                if kind == "text":
                    prompt = body.get("prompt")
                    if isinstance(prompt, list) and prompt and all(isinstance(t, int) for t in prompt):
                        ids = list(prompt)
                    elif isinstance(prompt, str):
                        ids = srv._encode(prompt)
                    elif isinstance(prompt, list) and prompt and all(isinstance(x, str) for x in prompt):
                        ids = [srv._encode(x) for x in prompt]  # a batch of prompts
                    elif isinstance(prompt, list) and prompt and all(
                            isinstance(x, list) and x and all(isinstance(t, int) for t in x) for x in prompt):
                        ids = [list(x) for x in prompt]
                    else:
                        raise ValueError("prompt must be a string, a list of strings or token id list(s)")
                    if ids and isinstance(ids[0], list) and body.get("stream"):
                        raise ValueError("a batch of prompts is not supported with stream")
                    params = _params(body)
                elif kind == "chat":
                    tools = tool_setup(body)
                    msgs = body.get("messages")
                    if tools is not None and isinstance(msgs, list):
                        msgs = [{"role": "system", "content": tools["prompt"]}] + list(msgs)
                    ids = srv._chat_prompt(msgs)
                    params = _params(body)
                    if tools is not None and tools["schema"] is not None:  # a tool call is required
                        params.json_schema, params.json_mode = tools["schema"], True
                else:
                    if body.get("messages") is not None:
                        ids = srv._chat_prompt(body["messages"])
                    else:
                        inp = body.get("input", body.get("prompt"))
                        if isinstance(inp, list):
                            ids = srv._chat_prompt(inp)
                        elif isinstance(inp, str):
                            ids = srv._encode(inp)
                        else:
                            raise ValueError("input (or prompt / messages) is required")
                    params = _params(body, "max_output_tokens")
                stops = srv._stops(body)
                n_choices = int(body.get("n", 1) or 1)
                if not 1 <= n_choices <= 16:
                    raise ValueError("n must be between 1 and 16")
                if body.get("stream"):
                    if n_choices > 1:
                        raise ValueError("n > 1 is not supported with stream")
                    if kind == "chat" and body.get("tools"):
                        raise ValueError("stream with tools is not supported; send stream=false")
                    so = body.get("stream_options") or {}
                    inc = bool(so.get("include_usage")) if isinstance(so, dict) else False
                    return srv._sse(srv._stream(ids, params, stops, kind, model, include_usage=inc))
                out = await srv._complete(ids, params, stops, kind, model, n_choices)
                if kind == "chat" and body.get("tools"):
                    _tool_calls(out, body)
                return JSONResponse(out)
            except ValueError as e:
                return _err(400, str(e))
            except Overloaded as e:  # admission control: queue full
                return _err(503, str(e), "overloaded_error")
            except Exception as e:  # engine failure
                return _err(500, f"{type(e).__name__}: {e}", "server_error")

        @app.post("/v1/embeddings")
        async def embeddings(request: Request):
            lim = srv._limit(request)
            if lim is not None:
                return lim
            try:
                body = await srv._body(request)
                inp = body.get("input")
                if isinstance(inp, str):
                    batch = [srv._encode(inp)]
                elif isinstance(inp, list) and inp and all(isinstance(t, int) for t in inp):
                    batch = [list(inp)]
                elif isinstance(inp, list) and inp and all(isinstance(x, str) for x in inp):
                    batch = [srv._encode(x) for x in inp]
                elif isinstance(inp, list) and inp and all(isinstance(x, list) for x in inp):
                    batch = [list(x) for x in inp]
                else:
                    raise ValueError("input must be a string, a list of strings or token-id list(s)")
                if any(not b for b in batch) or any(t < 0 or t >= srv.engine.cfg.vocab for b in batch for t in b):
                    raise ValueError("input token ids out of range")
                if not hasattr(srv.aengine, "call"):
                    raise ValueError("embeddings are not served by this front end")
                vecs = await srv.aengine.call(lambda eng: eng.embed(batch))
            except ValueError as e:
                return _err(400, str(e))
            except NotImplementedError as e:
                return _err(400, str(e))
            except Exception as e:  # engine failure
                return _err(500, f"{type(e).__name__}: {e}", "server_error")
            n_tok = sum(len(b) for b in batch)
            return JSONResponse({"object": "list", "model": body.get("model") or srv.model_id,
                                 "data": [{"object": "embedding", "index": i, "embedding": v.tolist()}
                                          for i, v in enumerate(vecs)],
                                 "usage": {"prompt_tokens": n_tok, "total_tokens": n_tok}}, headers=CORS)

        @app.post("/tokenize")
        async def tokenize(request: Request):
            """llama.cpp-style: {"content": str, "add_special": bool} -> {"tokens": [ids]}."""
            try:
                body = await srv._body(request)
                text = body.get("content")
                if not isinstance(text, str):
                    raise ValueError("content must be a string")
                ids = srv.tok.encode(text, add_special=bool(body.get("add_special", False)))
            except ValueError as e:
                return _err(400, str(e))
            return JSONResponse({"tokens": ids}, headers=CORS)

        @app.post("/detokenize")
        async def detokenize(request: Request):
            """{"tokens": [ids]} -> {"content": str}."""
            try:
                body = await srv._body(request)
                ids = body.get("tokens")
                if not isinstance(ids, list) or not all(isinstance(t, int) and 0 <= t < srv.tok.vocab_size
                                                        for t in ids):
                    raise ValueError("tokens must be a list of token ids")
            except ValueError as e:
                return _err(400, str(e))
            return JSONResponse({"content": srv.tok.decode(ids)}, headers=CORS)

        @app.post("/v1/completions")
        async def completions(request: Request):
            return await handle(request, "text")

        @app.post("/v1/chat/completions")
        async def chat(request: Request):
            return await handle(request, "chat")

        @app.post("/v1/responses")
        async def responses(request: Request):
            return await handle(request, "resp")

        @app.api_route("/{path:path}", methods=["GET", "POST", "PUT", "DELETE"])
        async def not_found(path: str):
            return _err(404, "route not found; try /v1/models, /v1/responses, /v1/completions or /v1/chat/completions",
                        "not_found_error")

        return app


def serve(server: OpenAIServer, host: str = "0.0.0.0", port: int = 8000) -> None:
    import uvicorn

    uvicorn.run(server.app, host=host, port=port, log_level="info")
