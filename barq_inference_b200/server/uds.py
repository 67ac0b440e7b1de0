"""Unix-domain-socket streaming server and client.

Parity: ``InferenceServer`` / ``InferenceClient`` (``advanced/src/uds_server.rs:18-395``).  Wire format
(kept identical): each frame is a 4-byte big-endian length followed by a UTF-8 JSON object.  A
request ``{"id", "prompt", "max_tokens", "temperature"}`` is answered by a stream of
``{"id", "text", "tokens_generated", "ttft_ms", "total_time_ms", "done"}`` frames, one per generated
token, the last with ``done: true``.  Requests from all connections share the continuous-batching
engine (what the reference's unreachable ``cmd_server_batch`` intended, ``cli/src/main.rs:1045-1158``).
Sampling uses top-k 40 / top-p 0.95 like the reference's handler.  Errors are reported as a final
frame with ``done: true`` and an ``error`` field.

Additive fields (a client of the reference's protocol neither sends nor needs them): a request may
carry ``messages`` (OpenAI chat turns, rendered with the server's chat template) instead of
``prompt``, the OpenAI sampling fields (``top_k``, ``top_p``, ``min_p``, ``seed``, penalties,
``response_format``, ``grammar``) and ``tools`` / ``tool_choice``; the final frame adds
``prompt_tokens``, ``finish_reason`` and, when the reply is a call of one of the tools,
``tool_call`` ({"name", "arguments"}); with ``logprobs`` / ``top_logprobs`` every token frame
carries ``logprobs`` = [{token, bytes, logprob, top: [{token, bytes, logprob}, ...]}].  A request ``{"id", "embeddings": input}`` (a string, a list
of strings, token ids or lists of token ids) is answered by one frame ``{"id", "embeddings":
[[...]], "prompt_tokens", "done": true}``; a request ``{"id", "health": true}`` by one frame with
``healthy``, ``last_error`` and ``kv_usage``; ``{"id", "metrics": true}`` by one frame whose
``prometheus`` member is the engine-side metrics text; ``{"id", "tokenize": text}`` /
``{"id", "detokenize": ids}`` by one frame with ``tokens`` / ``content``.  A client that disconnects mid-stream has its request
aborted in the engine.
"""
from __future__ import annotations

import json
import os
import socket
import socketserver
import struct
import threading
import time
from collections import OrderedDict

from ..tokenizer import ChatTemplate, StreamDecoder
from .chat_tools import normalize_messages, tool_call_of, tool_names, tool_setup
from .metrics import InferenceMetrics
from .request_params import sampling_params_from_request

MAX_FRAME = 16 << 20


def send_frame(sock: socket.socket, obj: dict) -> None:
    data = json.dumps(obj).encode("utf-8")
    sock.sendall(struct.pack(">I", len(data)) + data)


def _recv_exact(sock: socket.socket, n: int) -> bytes | None:
    buf = bytearray()
    while len(buf) < n:
        chunk = sock.recv(n - len(buf))
        if not chunk:
            return None
        buf += chunk
    return bytes(buf)


def recv_frame(sock: socket.socket) -> dict | None:
    head = _recv_exact(sock, 4)
    if head is None:
        return None
    (n,) = struct.unpack(">I", head)
    if n > MAX_FRAME:
        raise ValueError(f"frame of {n} bytes exceeds {MAX_FRAME}")
    body = _recv_exact(sock, n)
    if body is None:
        return None
    return json.loads(body.decode("utf-8"))


class UDSServer:
    def __init__(self, aengine, tokenizer, socket_path: str = "/tmp/barq-inference.sock", queue_size: int = 100,
                 metrics=None, chat_template: ChatTemplate | None = None):
        self.ae = aengine
        # per-request counters / TTFT: served by the metrics port and by {"metrics": true} frames
        self.metrics = metrics if metrics is not None else InferenceMetrics()
        self.tok = tokenizer
        self.template = chat_template or ChatTemplate("generic")
        # recent prompt texts -> token ids (repeated system prompts and retries skip the tokenizer;
        # the role of the reference's prompt-processing cache)
        self._tok_cache: OrderedDict[str, tuple[int, ...]] = OrderedDict()
        self._tok_lock = threading.Lock()
        self.tok_cache_size = 1024
        self.tok_cache_hits = 0
        self.path = socket_path
        self.sem = threading.BoundedSemaphore(queue_size)
        self._server = None

    def _encode(self, text: str, add_special: bool = True) -> list[int]:
        key = (text, add_special)
        with self._tok_lock:
            hit = self._tok_cache.get(key)
            if hit is not None:
                self._tok_cache.move_to_end(key)
                self.tok_cache_hits += 1
                return list(hit)
        ids = self.tok.encode(text, add_special=add_special)
        with self._tok_lock:
            self._tok_cache[key] = tuple(ids)
            if len(self._tok_cache) > self.tok_cache_size:
                self._tok_cache.popitem(last=False)
        return ids

    def _prompt_ids(self, req: dict, tools: dict | None = None) -> list[int]:
        msgs = req.get("messages")
        if msgs is not None:
            msgs = normalize_messages(msgs)
            if tools is not None:
                msgs = [{"role": "system", "content": tools["prompt"]}] + msgs
            text = self.template.render(msgs, add_generation_prompt=True)
            bos = getattr(self.template, "bos_token", "") or "\0"
            return self._encode(text, add_special=not text.startswith(bos))
        if tools is not None:
            raise ValueError("tools need chat messages")
        prompt = req["prompt"]
        if isinstance(prompt, list):
            return [int(t) for t in prompt]
        return self._encode(str(prompt))

    def handle_request(self, conn: socket.socket, req: dict) -> None:
        t0 = time.perf_counter()
        rid = str(req.get("id", ""))
        if "embeddings" in req:
            self._embed(conn, req, rid, t0)
            return
        if req.get("health"):
            send_frame(conn, self._health(rid))
            return
        if "tokenize" in req or "detokenize" in req:
            send_frame(conn, self._tokenize(req, rid))
            return
        if req.get("metrics"):
            eng = getattr(self.ae, "engine", None)
            send_frame(conn, {"id": rid, "text": "", "tokens_generated": 0, "ttft_ms": 0, "total_time_ms": 0,
                              "done": True, "prometheus": self.metrics.prometheus(eng)})
            return
        try:
            tools = tool_setup(req)
            ids = self._prompt_ids(req, tools)
            params = sampling_params_from_request(req)
            if tools is not None and tools["schema"] is not None:  # a tool call is required
                params.json_schema, params.json_mode = tools["schema"], True
        except Exception as e:  # noqa: BLE001 - any failure ends the stream with an error frame
            send_frame(conn, {"id": rid, "text": "", "tokens_generated": 0, "ttft_ms": 0, "total_time_ms": 0,
                              "done": True, "error": f"bad request: {e}"})
            return
        dec = StreamDecoder(self.tok)
        n, ttft, text = 0, None, []
        guard = self.metrics.begin() if self.metrics is not None else None
        gen = self.ae.generate_blocking(ids, params, rid)
        try:
            for item in gen:
                now = time.perf_counter()
                if item.token is None:
                    if guard is not None:
                        guard.complete(len(ids), n)
                        guard = None
                    tail = dec.flush()
                    last = {"id": rid, "text": tail, "tokens_generated": n, "ttft_ms": int(ttft or 0),
                            "total_time_ms": int((now - t0) * 1e3), "done": True, "prompt_tokens": len(ids),
                            "finish_reason": item.finish_reason or "stop"}
                    if tools is not None:
                        call = tool_call_of("".join(text) + tail, tool_names(req))
                        if call is not None:
                            last["tool_call"], last["finish_reason"] = call, "tool_calls"
                    send_frame(conn, last)
                    return
                n += 1
                if ttft is None:
                    ttft = (now - t0) * 1e3
                    if guard is not None:
                        guard.first_token()
                piece = dec.push(item.token)
                if tools is not None:
                    text.append(piece)
                fr = {"id": rid, "text": piece, "tokens_generated": n, "ttft_ms": int(ttft),
                      "total_time_ms": int((now - t0) * 1e3), "done": False}
                if params.logprobs:
                    e = self._lp_entry(item, n - 1, params)
                    if e is not None:
                        fr["logprobs"] = [e]
                send_frame(conn, fr)
        except OSError:  # the client went away mid-stream: closing the iterator aborts the request
            gen.close()
        except Exception as e:  # noqa: BLE001 - a failed request still gets its final frame
            if guard is not None:
                guard.fail()
                guard = None
            try:
                send_frame(conn, {"id": rid, "text": "", "tokens_generated": n, "ttft_ms": 0,
                                  "total_time_ms": int((time.perf_counter() - t0) * 1e3), "done": True,
                                  "error": str(e)})
            except OSError:
                pass
        finally:
            if guard is not None:  # client went away mid-stream
                guard.fail()

    def _tokenize(self, req: dict, rid: str) -> dict:
        """{"tokenize": text[, "add_special"]} -> {"tokens"}; {"detokenize": ids} -> {"content"}."""
        out = {"id": rid, "text": "", "tokens_generated": 0, "ttft_ms": 0, "total_time_ms": 0, "done": True}
        try:
            if "tokenize" in req:
                if not isinstance(req["tokenize"], str):
                    raise ValueError("tokenize takes a string")
                out["tokens"] = self.tok.encode(req["tokenize"], add_special=bool(req.get("add_special", False)))
            else:
                ids = req["detokenize"]
                if not isinstance(ids, list) or not all(isinstance(t, int) and 0 <= t < self.tok.vocab_size
                                                        for t in ids):
                    raise ValueError("detokenize takes a list of token ids")
                out["content"] = self.tok.decode(ids)
        except ValueError as e:
            out["error"] = f"bad request: {e}"
        return out

    def _health(self, rid: str) -> dict:
        """{"healthy", "last_error", "kv_usage"} of the engine behind this server (one frame)."""
        eng = getattr(self.ae, "engine", None)
        blocks = getattr(eng, "blocks", None)
        used = blocks.n_used / blocks.num_blocks if blocks is not None and blocks.num_blocks else 0.0
        return {"id": rid, "text": "", "tokens_generated": 0, "ttft_ms": 0, "total_time_ms": 0, "done": True,
                "healthy": bool(getattr(self.ae, "healthy", True)), "last_error": getattr(self.ae, "last_error", None),
                "kv_usage": used}

    def _lp_entry(self, item, idx: int, params) -> dict | None:
        """{token, bytes, logprob, top: [{token, bytes, logprob}]} of the idx-th generated token, from
        the engine's per-sequence record; None for an end-of-sequence token or when nothing was
        recorded."""
        cfg = getattr(getattr(self.ae, "engine", None), "cfg", None) or getattr(self.ae, "cfg", None)
        if cfg is not None and item.token in cfg.eos_ids and not params.ignore_eos:
            return None
        lps = getattr(item.seq, "logprobs", None)
        if not lps or idx >= len(lps):
            return None
        tops = getattr(item.seq, "top_logprobs", None) or []

        def tok(tid):
            b = self.tok.token_bytes(tid) if hasattr(self.tok, "token_bytes") else self.tok.decode([tid]).encode()
            return {"token": b.decode("utf-8", errors="replace"), "bytes": list(b)}

        return {**tok(item.token), "logprob": float(lps[idx]),
                "top": [{**tok(a), "logprob": float(v)} for a, v in (tops[idx] if idx < len(tops) else [])]}

    def _embed(self, conn: socket.socket, req: dict, rid: str, t0: float) -> None:
        """One frame with the mean-pooled embeddings of the request's inputs (or an error frame)."""
        def frame(**kw):
            return {"id": rid, "text": "", "tokens_generated": 0, "ttft_ms": 0,
                    "total_time_ms": int((time.perf_counter() - t0) * 1e3), "done": True, **kw}

        try:
            inp = req["embeddings"]
            if isinstance(inp, str):
                batch = [self.tok.encode(inp)]
            elif isinstance(inp, list) and inp and all(isinstance(t, int) for t in inp):
                batch = [list(inp)]
            elif isinstance(inp, list) and inp and all(isinstance(x, str) for x in inp):
                batch = [self.tok.encode(x) for x in inp]
            elif isinstance(inp, list) and inp and all(isinstance(x, list) for x in inp):
                batch = [[int(t) for t in x] for x in inp]
            else:
                raise ValueError("embeddings input must be a string, a list of strings or token-id list(s)")
            if any(not b for b in batch):
                raise ValueError("empty embeddings input")
            if not hasattr(self.ae, "call_sync"):
                raise ValueError("embeddings are not served by this engine front")
            vecs = self.ae.call_sync(lambda eng: eng.embed(batch))
        except Exception as e:  # noqa: BLE001 - reported in the frame
            send_frame(conn, frame(error=f"bad request: {e}" if isinstance(e, (ValueError, KeyError)) else str(e)))
            return
        send_frame(conn, frame(embeddings=[v.tolist() for v in vecs], prompt_tokens=sum(len(b) for b in batch)))

    def start(self, background: bool = True):
        if os.path.exists(self.path):
            os.unlink(self.path)
        srv = self

        class Handler(socketserver.BaseRequestHandler):
            def handle(self):
                conn = self.request
                while True:
                    try:
                        req = recv_frame(conn)
                    except (ValueError, json.JSONDecodeError) as e:
                        send_frame(conn, {"id": "", "text": "", "tokens_generated": 0, "ttft_ms": 0,
                                          "total_time_ms": 0, "done": True, "error": str(e)})
                        return
                    if req is None:
                        return
                    if not srv.sem.acquire(blocking=False):
                        send_frame(conn, {"id": str(req.get("id", "")), "text": "", "tokens_generated": 0,
                                          "ttft_ms": 0, "total_time_ms": 0, "done": True, "error": "queue full"})
                        continue
                    try:
                        srv.handle_request(conn, req)
                    finally:
                        srv.sem.release()

        class Server(socketserver.ThreadingMixIn, socketserver.UnixStreamServer):
            daemon_threads = True

        self._server = Server(self.path, Handler)
        # owner-only by default: any local user who can connect can generate (BARQ_SOCKET_MODE=660
        # shares it with the group, e.g. a front end running as another user)
        os.chmod(self.path, int(os.environ.get("BARQ_SOCKET_MODE", "600"), 8))
        if background:
            threading.Thread(target=self._server.serve_forever, daemon=True).start()
        else:
            self._server.serve_forever()
        return self

    def stop(self):
        if self._server is not None:
            self._server.shutdown()
            self._server.server_close()
        if os.path.exists(self.path):
            os.unlink(self.path)


class UDSClient:
    def __init__(self, socket_path: str = "/tmp/barq-inference.sock"):
        self.sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self.sock.connect(socket_path)

    def stream(self, prompt, max_tokens: int = 128, temperature: float = 0.8, rid: str = "req"):
        send_frame(self.sock, {"id": rid, "prompt": prompt, "max_tokens": max_tokens, "temperature": temperature})
        while True:
            fr = recv_frame(self.sock)
            if fr is None:
                return
            yield fr
            if fr.get("done"):
                return

    def query(self, what: str) -> dict:
        """One-frame engine query: ``"health"`` -> {healthy, last_error, kv_usage}, ``"metrics"`` ->
        {prometheus}."""
        send_frame(self.sock, {"id": what, what: True})
        return recv_frame(self.sock) or {}

    def close(self):
        self.sock.close()
