"""The native HTTP front end (``barq-http``, ``csrc/client/barq_http.cpp``) on CPU.

A scripted UDS server stands in for the engine and records the frames the front end sends, so the
tests check both sides of the translation: OpenAI request -> UDS request, UDS frames -> OpenAI
responses / SSE chunks.  The last test runs the front end against the real UDS server and the CPU
engine and compares its greedy text with the UDS client's."""
import http.client
import json
import os
import shutil
import socket
import subprocess
import threading
import time

import pytest

from barq_inference_b200.server.uds import recv_frame, send_frame

pytestmark = pytest.mark.skipif(shutil.which("g++") is None and shutil.which("c++") is None,
                                reason="no C++ compiler")

SCRIPTS = {
    # prompt / last message content -> (frame texts, final extras) or an error string
    "hello": (["Hel", "lo", " wor", "ld"], {"prompt_tokens": 3, "finish_reason": "length"}),
    "stop": (["ab", "c<e", "nd>tail", "more"], {"prompt_tokens": 2, "finish_reason": "length"}),
    "near": (["x<e", "y"], {"prompt_tokens": 1, "finish_reason": "stop"}),
    "utf8": (["é", "\U0001F600", "\"q\"\n"], {"prompt_tokens": 4, "finish_reason": "stop"}),
    "slow": (["s"] * 200, {"prompt_tokens": 1, "finish_reason": "length"}),
    "queue": "queue full",
    "badreq": "bad request: temperature must be a number",
    "boom": "RuntimeError: engine exploded",
}


class FakeEngine:
    def __init__(self, path):
        self.path = path
        self.requests = []
        self.aborted = []
        self.healthy = True
        self.lock = threading.Lock()
        self.sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self.sock.bind(path)
        self.sock.listen(64)
        threading.Thread(target=self._accept, daemon=True).start()

    def _accept(self):
        while True:
            try:
                conn, _ = self.sock.accept()
            except OSError:
                return
            threading.Thread(target=self._serve, args=(conn,), daemon=True).start()

    def _serve(self, conn):
        try:
            req = recv_frame(conn)
            if req is None:  # a connect-and-close probe
                return
            if req.get("metrics"):
                send_frame(conn, {"id": req["id"], "text": "", "done": True,
                                  "prometheus": "# TYPE barq_requests_total counter\nbarq_requests_total 7\n"})
                return
            if req.get("health"):
                send_frame(conn, {"id": req["id"], "text": "", "done": True, "healthy": self.healthy,
                                  "last_error": None if self.healthy else "step failed", "kv_usage": 0.25})
                return
            with self.lock:
                self.requests.append(req)
            if "embeddings" in req:
                inp = req["embeddings"]
                n = len(inp) if isinstance(inp, list) and inp and not isinstance(inp[0], int) else 1
                send_frame(conn, {"id": req["id"], "text": "", "tokens_generated": 0, "ttft_ms": 0, "total_time_ms": 1,
                                  "done": True, "embeddings": [[0.5 + i, -1.25e-3, 1e-30] for i in range(n)],
                                  "prompt_tokens": 3 * n})
                return
            key = req.get("prompt")
            if key is None:
                key = req["messages"][-1]["content"]
            script = SCRIPTS.get(key if isinstance(key, str) else "hello", SCRIPTS["hello"])
            rid = req.get("id", "")
            if isinstance(script, str):
                send_frame(conn, {"id": rid, "text": "", "tokens_generated": 0, "ttft_ms": 0, "total_time_ms": 0,
                                  "done": True, "error": script})
                return
            texts, extra = script
            for i, t in enumerate(texts):
                if key == "slow":
                    time.sleep(0.01)
                send_frame(conn, {"id": rid, "text": t, "tokens_generated": i + 1, "ttft_ms": 1,
                                  "total_time_ms": 2, "done": False})
            last = {"id": rid, "text": "", "tokens_generated": len(texts), "ttft_ms": 1, "total_time_ms": 3,
                    "done": True, **extra}
            if req.get("tools"):
                last.update(tool_call={"name": "get_weather", "arguments": {"city": "Paris", "days": 2}},
                            finish_reason="tool_calls")
            send_frame(conn, last)
        except OSError:
            with self.lock:
                self.aborted.append(True)
        finally:
            conn.close()

    def close(self):
        self.sock.close()


def _start(sock_path, *extra):
    from barq_inference_b200.server.uds_native import build_http

    exe = build_http()
    p = subprocess.Popen([exe, "--socket", sock_path, "--host", "127.0.0.1", "--port", "0", "--model-id", "tiny-x",
                          "--quiet", *extra], stdout=subprocess.PIPE, stderr=subprocess.PIPE)
    line = p.stdout.readline().decode()
    assert "listening on 127.0.0.1:" in line, (line, p.stderr.read() if p.poll() is not None else b"")
    port = int(line.split("127.0.0.1:")[1].split()[0])
    return p, port


@pytest.fixture()
def gateway(tmp_path):
    eng = FakeEngine(str(tmp_path / "e.sock"))
    p, port = _start(eng.path)
    yield eng, port
    p.kill()
    p.wait()
    eng.close()


def _req(port, method, path, body=None, headers=None, raw=None):
    c = http.client.HTTPConnection("127.0.0.1", port, timeout=30)
    data = raw if raw is not None else (json.dumps(body).encode() if body is not None else None)
    c.request(method, path, body=data, headers={"Content-Type": "application/json", **(headers or {})})
    r = c.getresponse()
    out = r.status, dict(r.getheaders()), r.read()
    c.close()
    return out


def _metric(text: str, name: str) -> float:
    return float(next(line.split()[1] for line in text.splitlines() if line.startswith(name + " ")))


def _events(raw: bytes):
    evs = [e[len("data: "):] for e in raw.decode().split("\n\n") if e.startswith("data: ")]
    assert evs[-1] == "[DONE]"
    return [json.loads(e) for e in evs[:-1]]


def test_info_models_health_and_cors(gateway, tmp_path):
    eng, port = gateway
    st, h, b = _req(port, "GET", "/v1/models")
    assert st == 200 and json.loads(b)["data"][0]["id"] == "tiny-x"
    st, _, b = _req(port, "GET", "/v1/models/tiny-x")
    assert st == 200 and json.loads(b)["id"] == "tiny-x" and json.loads(b)["object"] == "model"
    assert _req(port, "GET", "/v1/models/other")[0] == 404
    assert h["Access-Control-Allow-Origin"] == "*"
    st, _, b = _req(port, "GET", "/")
    assert st == 200 and "/v1/chat/completions" in json.loads(b)["endpoints"]
    st, _, b = _req(port, "GET", "/health")
    assert st == 200 and json.loads(b)["status"] == "ok" and json.loads(b)["kv_usage"] == 0.25
    eng.healthy = False
    st, _, b = _req(port, "GET", "/health")
    assert st == 503 and json.loads(b)["status"] == "degraded" and json.loads(b)["last_error"] == "step failed"
    eng.healthy = True
    st, h, b = _req(port, "OPTIONS", "/v1/chat/completions")
    assert st == 204 and "POST" in h["Access-Control-Allow-Methods"] and b == b""
    st, _, b = _req(port, "GET", "/nope")
    assert st == 404 and json.loads(b)["error"]["type"] == "not_found_error"
    assert "try /v1/models" in json.loads(b)["error"]["message"]
    st, _, _ = _req(port, "GET", "/v1/completions")
    assert st == 405
    # an engine socket that does not exist: health 503, generation 502
    p, port2 = _start(str(tmp_path / "none.sock"))
    try:
        assert _req(port2, "GET", "/health")[0] == 503
        st, _, b = _req(port2, "POST", "/v1/completions", {"prompt": "hello"})
        assert st == 502 and json.loads(b)["error"]["type"] == "engine_unavailable_error"
    finally:
        p.kill()
        p.wait()


def test_completion_translation_both_ways(gateway):
    eng, port = gateway
    body = {"prompt": "hello", "max_tokens": 7, "temperature": 0.25, "top_k": 5, "top_p": 0.5, "seed": 11,
            "min_p": 0.1, "repetition_penalty": 1.1, "response_format": {"type": "json_object"}, "grammar": "root ::= \"a\"",
            "unknown_field": [1, 2]}
    st, h, b = _req(port, "POST", "/v1/completions", body, headers={"x-request-id": "abc-123"})
    assert st == 200, b
    assert h["x-request-id"] == "abc-123"
    out = json.loads(b)
    assert out["object"] == "text_completion" and out["id"].startswith("cmpl-") and out["model"] == "tiny-x"
    assert out["choices"] == [{"index": 0, "text": "Hello world", "finish_reason": "length", "logprobs": None}]
    assert out["usage"] == {"prompt_tokens": 3, "completion_tokens": 4, "total_tokens": 7}
    sent = eng.requests[-1]
    assert sent == {"id": "abc-123", "prompt": "hello", "max_tokens": 7, "temperature": 0.25, "top_k": 5,
                    "top_p": 0.5, "min_p": 0.1, "seed": 11, "repetition_penalty": 1.1,
                    "response_format": {"type": "json_object"}, "grammar": "root ::= \"a\""}
    # token-id prompts pass through; the model field is echoed
    st, _, b = _req(port, "POST", "/v1/completions", {"prompt": [1, 2, 3], "model": "m2"})
    assert st == 200 and json.loads(b)["model"] == "m2" and eng.requests[-1]["prompt"] == [1, 2, 3]
    # non-ASCII text and escapes survive both hops
    st, _, b = _req(port, "POST", "/v1/completions", {"prompt": "utf8"})
    assert json.loads(b)["choices"][0]["text"] == "é\U0001F600\"q\"\n"


def test_chat_and_responses_routes(gateway):
    eng, port = gateway
    msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hello"}]
    st, _, b = _req(port, "POST", "/v1/chat/completions", {"messages": msgs, "max_tokens": 4})
    out = json.loads(b)
    assert st == 200 and out["object"] == "chat.completion" and out["id"].startswith("chatcmpl-")
    assert out["choices"][0]["message"] == {"role": "assistant", "content": "Hello world"}
    assert eng.requests[-1]["messages"] == msgs and "prompt" not in eng.requests[-1]
    st, _, b = _req(port, "POST", "/v1/responses", {"input": "hello", "max_output_tokens": 9})
    out = json.loads(b)
    assert st == 200 and out["object"] == "response" and out["output"] == "Hello world"
    assert eng.requests[-1]["prompt"] == "hello" and eng.requests[-1]["max_tokens"] == 9
    st, _, b = _req(port, "POST", "/v1/responses", {"input": msgs})
    assert st == 200 and eng.requests[-1]["messages"] == msgs
    # n choices: one engine request per choice, seeds offset, usage summed
    st, _, b = _req(port, "POST", "/v1/chat/completions", {"messages": msgs, "n": 3, "seed": 5})
    out = json.loads(b)
    assert [c["index"] for c in out["choices"]] == [0, 1, 2] and out["usage"]["completion_tokens"] == 12
    assert sorted(r.get("seed") for r in eng.requests[-3:]) == [5, 6, 7]  # concurrent engine requests


def test_batch_of_prompts(gateway):
    eng, port = gateway
    st, _, b = _req(port, "POST", "/v1/completions", {"prompt": ["hello", "utf8"], "n": 2})
    out = json.loads(b)
    assert st == 200 and [c["index"] for c in out["choices"]] == [0, 1, 2, 3]
    assert [c["text"] for c in out["choices"]] == ["Hello world", "Hello world", "é\U0001F600\"q\"\n", "é\U0001F600\"q\"\n"]
    assert out["usage"]["prompt_tokens"] == 3 + 4  # each prompt once (the scripted engine's counts)
    assert _req(port, "POST", "/v1/completions", {"prompt": ["a", "b"], "stream": True})[0] == 400
    assert _req(port, "POST", "/v1/completions", {"prompt": [[1, 2], [3]]})[0] == 200


def test_streams(gateway):
    eng, port = gateway
    st, h, b = _req(port, "POST", "/v1/chat/completions",
                    {"messages": [{"role": "user", "content": "hello"}], "stream": True,
                     "stream_options": {"include_usage": True}})
    assert st == 200 and h["Content-Type"] == "text/event-stream"
    ev = _events(b)
    assert ev[0]["choices"][0]["delta"] == {"role": "assistant"}
    assert "".join(e["choices"][0]["delta"].get("content", "") for e in ev[1:-1]) == "Hello world"
    assert ev[-2]["choices"][0]["finish_reason"] == "length"
    assert ev[-1]["choices"] == [] and ev[-1]["usage"]["total_tokens"] == 7
    assert all(e["object"] == "chat.completion.chunk" for e in ev)
    st, _, b = _req(port, "POST", "/v1/completions", {"prompt": "hello", "stream": True})
    ev = _events(b)
    assert "".join(e["choices"][0]["text"] for e in ev) == "Hello world" and ev[-1]["choices"][0]["finish_reason"]
    st, _, b = _req(port, "POST", "/v1/responses", {"input": "hello", "stream": True})
    assert "".join(e["output"] for e in _events(b)) == "Hello world"


def test_streams_are_chunk_encoded_and_keep_the_connection(gateway):
    eng, port = gateway
    c = http.client.HTTPConnection("127.0.0.1", port, timeout=30)
    for _ in range(2):  # two streamed requests, then a plain one, on one connection
        c.request("POST", "/v1/completions", body=json.dumps({"prompt": "hello", "stream": True}),
                  headers={"Content-Type": "application/json"})
        r = c.getresponse()
        assert r.status == 200 and r.getheader("Transfer-Encoding") == "chunked"
        assert "".join(e["choices"][0]["text"] for e in _events(r.read())) == "Hello world"
    c.request("POST", "/v1/completions", body=json.dumps({"prompt": "hello"}), headers={"Content-Type": "application/json"})
    assert json.loads(c.getresponse().read())["choices"][0]["text"] == "Hello world"
    c.close()
    # an HTTP/1.0 client gets a close-delimited stream
    s = socket.create_connection(("127.0.0.1", port))
    body = json.dumps({"prompt": "hello", "stream": True}).encode()
    s.sendall(b"POST /v1/completions HTTP/1.0\r\nContent-Length: " + str(len(body)).encode() + b"\r\n\r\n" + body)
    data = b""
    while True:
        chunk = s.recv(65536)
        if not chunk:
            break
        data += chunk
    s.close()
    head, _, rest = data.partition(b"\r\n\r\n")
    assert b"Transfer-Encoding" not in head and b"Connection: close" in head
    assert "".join(e["choices"][0]["text"] for e in _events(rest)) == "Hello world"


def test_expect_100_continue(gateway):
    """A client that waits for "100 Continue" before its body (curl, for bodies over 1 KB) gets it
    right away."""
    eng, port = gateway
    body = json.dumps({"prompt": "hello", "pad": "x" * 2000}).encode()
    s = socket.create_connection(("127.0.0.1", port), timeout=5)
    s.sendall(b"POST /v1/completions HTTP/1.1\r\nContent-Type: application/json\r\nExpect: 100-continue\r\n"
              b"Content-Length: " + str(len(body)).encode() + b"\r\nConnection: close\r\n\r\n")
    assert s.recv(64).startswith(b"HTTP/1.1 100 Continue")  # before any body byte was sent
    s.sendall(body)
    data = b""
    while True:
        chunk = s.recv(65536)
        if not chunk:
            break
        data += chunk
    s.close()
    assert data.startswith(b"HTTP/1.1 200") and b"Hello world" in data


def test_stop_strings_are_never_sent(gateway):
    eng, port = gateway
    st, _, b = _req(port, "POST", "/v1/completions", {"prompt": "stop", "stop": ["<end>", "zz"], "stream": True})
    ev = _events(b)
    texts = [e["choices"][0]["text"] for e in ev]
    assert "".join(texts) == "abc" and all("<" not in t for t in texts)
    assert ev[-1]["choices"][0]["finish_reason"] == "stop"
    st, _, b = _req(port, "POST", "/v1/completions", {"prompt": "stop", "stop": "<end>"})
    assert json.loads(b)["choices"][0] == {"index": 0, "text": "abc", "finish_reason": "stop", "logprobs": None}
    # a held-back prefix that never completes the stop string is released at the end
    st, _, b = _req(port, "POST", "/v1/completions", {"prompt": "near", "stop": ["<end>"], "stream": True})
    assert "".join(e["choices"][0]["text"] for e in _events(b)) == "x<ey"


def test_errors(gateway):
    eng, port = gateway
    cases = [
        (dict(raw=b"{not json"), 400, "not valid JSON"),
        (dict(body=[1, 2]), 400, "JSON object"),
        (dict(body={"max_tokens": 3}), 400, "prompt must be"),
        (dict(body={"prompt": "hello", "max_tokens": 0}), 400, "max_tokens"),
        (dict(body={"prompt": "hello", "temperature": "hot"}), 400, "temperature must be a number"),
        (dict(body={"prompt": "hello", "n": 17}), 400, "n must be"),
        (dict(body={"prompt": "hello", "n": 2, "stream": True}), 400, "not supported with stream"),
        (dict(body={"prompt": "hello", "stop": 5}), 400, "stop must be"),
        (dict(body={"prompt": "queue"}), 503, "queue full"),
        (dict(body={"prompt": "queue", "stream": True}), 503, "queue full"),
        (dict(body={"prompt": "badreq"}), 400, "bad request"),
        (dict(body={"prompt": "boom"}), 500, "engine exploded"),
    ]
    for kw, status, text in cases:
        st, h, b = _req(port, "POST", "/v1/completions", **kw)
        assert st == status, (kw, st, b)
        assert text in json.loads(b)["error"]["message"], (kw, b)
    st, _, b = _req(port, "POST", "/v1/chat/completions", {"messages": []})
    assert st == 400
    st, _, b = _req(port, "POST", "/v1/chat/completions",
                    {"messages": [{"role": "user", "content": "x"}], "tools": [{"function": {"name": "f"}}],
                     "stream": True})
    assert st == 400 and "tools" in json.loads(b)["error"]["message"]
    st, _, b = _req(port, "POST", "/v1/chat/completions", {"messages": [{"role": "user", "content": "x"}], "tools": 3})
    assert st == 400
    # oversized headers and bodies are refused before any engine call
    n_before = len(eng.requests)
    st, _, _ = _req(port, "POST", "/v1/completions", raw=b"{}", headers={"X-Big": "a" * 40000})
    assert st == 431
    s = socket.create_connection(("127.0.0.1", port))
    s.sendall(b"POST /v1/completions HTTP/1.1\r\nContent-Length: 99999999\r\n\r\n")
    assert s.recv(100).startswith(b"HTTP/1.1 413")
    s.close()
    s = socket.create_connection(("127.0.0.1", port))
    s.sendall(b"garbage\r\n\r\n")
    assert s.recv(100).startswith(b"HTTP/1.1 400")
    s.close()
    assert len(eng.requests) == n_before
    st, _, b = _req(port, "GET", "/metrics")
    m = b.decode()
    assert "barq_http_requests_total" in m and "barq_http_client_errors_total" in m
    assert _metric(m, "barq_requests_total") == 7  # the engine's own metrics follow the front end's
    assert _metric(m, "barq_http_server_errors_total") >= 3 and _metric(m, "barq_http_client_errors_total") >= 10


def test_tools_and_embeddings(gateway):
    eng, port = gateway
    tools = [{"type": "function", "function": {"name": "get_weather", "parameters": {"type": "object"}}}]
    body = {"messages": [{"role": "user", "content": "hello"}], "tools": tools, "tool_choice": "required"}
    st, _, b = _req(port, "POST", "/v1/chat/completions", body)
    out = json.loads(b)
    assert st == 200, b
    assert eng.requests[-1]["tools"] == tools and eng.requests[-1]["tool_choice"] == "required"
    ch = out["choices"][0]
    assert ch["finish_reason"] == "tool_calls" and ch["message"]["content"] is None
    call = ch["message"]["tool_calls"][0]
    assert call["type"] == "function" and call["function"]["name"] == "get_weather"
    assert json.loads(call["function"]["arguments"]) == {"city": "Paris", "days": 2}
    st, _, b = _req(port, "POST", "/v1/embeddings", {"input": ["a", "b"], "model": "e5"})
    out = json.loads(b)
    assert st == 200 and out["object"] == "list" and out["model"] == "e5"
    assert [d["index"] for d in out["data"]] == [0, 1] and out["data"][1]["embedding"] == [1.5, -1.25e-3, 1e-30]
    assert out["usage"] == {"prompt_tokens": 6, "total_tokens": 6}
    assert eng.requests[-1]["embeddings"] == ["a", "b"]
    assert _req(port, "POST", "/v1/embeddings", {"input": 5})[0] == 400
    assert _req(port, "GET", "/v1/embeddings")[0] == 405


def test_keep_alive_and_client_disconnect(gateway):
    eng, port = gateway
    c = http.client.HTTPConnection("127.0.0.1", port, timeout=30)
    for _ in range(3):  # three requests on one connection
        c.request("POST", "/v1/completions", body=json.dumps({"prompt": "hello"}),
                  headers={"Content-Type": "application/json"})
        r = c.getresponse()
        assert r.status == 200 and json.loads(r.read())["choices"][0]["text"] == "Hello world"
    c.close()
    # a streaming client that goes away: the front end closes its engine connection early
    s = socket.create_connection(("127.0.0.1", port))
    body = json.dumps({"prompt": "slow", "stream": True}).encode()
    s.sendall(b"POST /v1/completions HTTP/1.1\r\nContent-Type: application/json\r\nContent-Length: "
              + str(len(body)).encode() + b"\r\n\r\n" + body)
    assert s.recv(64).startswith(b"HTTP/1.1 200")
    s.close()
    deadline = time.time() + 20
    while time.time() < deadline and not eng.aborted:
        time.sleep(0.05)
    assert eng.aborted, "the engine connection stayed open after the client left"


def test_non_streamed_client_leaving_stops_the_generation(gateway):
    eng, port = gateway
    n0 = len(eng.aborted)
    s = socket.create_connection(("127.0.0.1", port))
    body = json.dumps({"prompt": "slow"}).encode()
    s.sendall(b"POST /v1/completions HTTP/1.1\r\nContent-Type: application/json\r\nContent-Length: "
              + str(len(body)).encode() + b"\r\n\r\n" + body)
    time.sleep(0.2)  # the engine is streaming into the front end
    s.close()
    deadline = time.time() + 20
    while time.time() < deadline and len(eng.aborted) == n0:
        time.sleep(0.05)
    assert len(eng.aborted) > n0, "the engine connection stayed open after the client left"


def test_graceful_stop_lets_streams_finish(tmp_path):
    import signal

    eng = FakeEngine(str(tmp_path / "e.sock"))
    p, port = _start(eng.path, "--drain-timeout", "30")
    try:
        s = socket.create_connection(("127.0.0.1", port))
        body = json.dumps({"prompt": "slow", "stream": True}).encode()
        s.sendall(b"POST /v1/completions HTTP/1.1\r\nContent-Type: application/json\r\nContent-Length: "
                  + str(len(body)).encode() + b"\r\n\r\n" + body)
        first = s.recv(64)
        assert first.startswith(b"HTTP/1.1 200")
        p.send_signal(signal.SIGTERM)
        data = first
        while True:
            chunk = s.recv(65536)
            if not chunk:
                break
            data += chunk
        s.close()
        assert data.rstrip().endswith(b"0")  # the chunk-encoded stream in flight completed: [DONE], last chunk
        assert b"data: [DONE]" in data
        assert data.count(b'"text":"s"') == 200
        assert p.wait(timeout=30) == 0
        with pytest.raises(OSError):
            socket.create_connection(("127.0.0.1", port), timeout=2).close()
    finally:
        if p.poll() is None:
            p.kill()
            p.wait()
        eng.close()


def test_rate_limit(tmp_path):
    eng = FakeEngine(str(tmp_path / "e.sock"))
    p, port = _start(eng.path, "--rpm", "2")
    try:
        codes = [_req(port, "POST", "/v1/completions", {"prompt": "hello"})[0] for _ in range(3)]
        assert codes == [200, 200, 429]
        st, _, b = _req(port, "POST", "/v1/completions", {"prompt": "hello"})
        assert st == 429 and json.loads(b)["error"]["type"] == "rate_limit_error"
        m = _req(port, "GET", "/metrics")[2].decode()
        assert _metric(m, "barq_http_rate_limited_total") == 2
    finally:
        p.kill()
        p.wait()
        eng.close()


def test_against_real_uds_server_and_cpu_engine(tmp_path):
    """Greedy text through barq-http equals the UDS client's for the same prompt; chat messages are
    rendered by the engine's template; usage counts match the tokenizer."""
    from barq_inference_b200.engine.cpu_engine import CPUEngine
    from barq_inference_b200.models import POLICIES, preset, random_tensors
    from barq_inference_b200.server.async_engine import AsyncEngine
    from barq_inference_b200.server.uds import UDSClient, UDSServer
    from barq_inference_b200.tokenizer import synthetic_tokenizer

    cfg = preset("tiny", n_layers=1, vocab=600, max_ctx=2048)
    eng = CPUEngine(cfg, random_tensors(cfg, POLICIES["tiny"], seed=0), max_model_len=2048)
    tok = synthetic_tokenizer(cfg.vocab)
    eng.tokenizer = tok  # token strings for grammar-constrained (tool call) sampling
    path = str(tmp_path / "real.sock")
    ae = AsyncEngine(eng)
    srv = UDSServer(ae, tok, path).start()
    p, port = _start(path)
    try:
        cl = UDSClient(path)
        want = "".join(f["text"] for f in cl.stream("hello world", max_tokens=8, temperature=0.0, rid="u"))
        cl.close()
        st, _, b = _req(port, "POST", "/v1/completions",
                        {"prompt": "hello world", "max_tokens": 8, "temperature": 0.0})
        out = json.loads(b)
        assert st == 200 and out["choices"][0]["text"] == want
        assert out["usage"]["prompt_tokens"] == len(tok.encode("hello world"))
        assert out["choices"][0]["finish_reason"] in ("length", "stop")
        st, _, b = _req(port, "POST", "/v1/chat/completions",
                        {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4, "temperature": 0.0,
                         "stream": True})
        ev = _events(b)
        assert st == 200 and ev[0]["choices"][0]["delta"] == {"role": "assistant"}
        st, _, b = _req(port, "POST", "/v1/completions", {"prompt": "x " * 2000, "max_tokens": 100})
        assert st == 400 and "max_model_len" in json.loads(b)["error"]["message"]
        # logprobs through the engine: one entry per generated token, greedy = the top alternative
        st, _, b = _req(port, "POST", "/v1/chat/completions",
                        {"messages": [{"role": "user", "content": "hi"}], "max_tokens": 5, "temperature": 0,
                         "logprobs": True, "top_logprobs": 2})
        out = json.loads(b)
        ents = out["choices"][0]["logprobs"]["content"]
        assert st == 200 and len(ents) == out["usage"]["completion_tokens"] - (out["choices"][0]["finish_reason"] == "stop")
        for e in ents:
            assert len(e["top_logprobs"]) == 2 and abs(e["logprob"] - e["top_logprobs"][0]["logprob"]) < 1e-5
        st, _, b = _req(port, "POST", "/v1/completions",
                        {"prompt": "hello", "max_tokens": 4, "temperature": 0, "logprobs": 1, "stream": True})
        evs = _events(b)
        toks = [t for ev in evs for t in ((ev["choices"][0].get("logprobs") or {}).get("tokens") or [])]
        assert "".join(toks) == "".join(ev["choices"][0]["text"] for ev in evs)
        m = _req(port, "GET", "/metrics")[2].decode()
        assert "barq_http_requests_total" in m and "barq_requests_total" in m
        st, _, b = _req(port, "POST", "/tokenize", {"content": "hello world", "add_special": True})
        assert st == 200 and json.loads(b)["tokens"] == tok.encode("hello world", add_special=True)
        st, _, b = _req(port, "POST", "/detokenize", {"tokens": json.loads(b)["tokens"]})
        assert st == 200 and json.loads(b)["content"] == tok.decode(tok.encode("hello world", add_special=True))
        assert _req(port, "POST", "/detokenize", {"tokens": [10 ** 9]})[0] == 400
        assert _req(port, "POST", "/tokenize", {"content": 5})[0] == 400
        # embeddings through the engine: one vector per input, same as the engine's own
        st, _, b = _req(port, "POST", "/v1/embeddings", {"input": ["hello", "world wide"]})
        out = json.loads(b)
        want = eng.embed([tok.encode("hello"), tok.encode("world wide")])
        assert st == 200 and len(out["data"]) == 2
        assert max(abs(a - float(b_)) for a, b_ in zip(out["data"][1]["embedding"], want[1].tolist())) < 1e-6
        # a required tool call: the engine constrains the reply to the function's schema
        tools = [{"type": "function", "function": {"name": "lookup", "parameters": {
            "type": "object", "properties": {"q": {"type": "string", "maxLength": 4}}, "required": ["q"]}}}]
        st, _, b = _req(port, "POST", "/v1/chat/completions",
                        {"messages": [{"role": "user", "content": "find"}], "tools": tools,
                         "tool_choice": "required", "max_tokens": 60, "temperature": 0})
        out = json.loads(b)
        assert st == 200, b
        calls = out["choices"][0]["message"].get("tool_calls")
        if out["choices"][0]["finish_reason"] != "length":  # a complete call within the token budget
            assert calls and calls[0]["function"]["name"] == "lookup"
            assert "q" in json.loads(calls[0]["function"]["arguments"])
    finally:
        p.kill()
        p.wait()
        srv.stop()
        ae.shutdown()


def test_cli_http_server_native_front_end(tmp_path):
    """``barq http-server --native-front-end``: the CLI serves HTTP through barq-http with the engine
    behind a private UDS socket."""
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    model = str(tmp_path / "tiny.gguf")
    r = subprocess.run([sys.executable, "-m", "barq_inference_b200.cli", "make-random-gguf", "--arch", "tiny",
                        "--layers", "1", "--output", model, "--device", "cpu"], cwd=root, capture_output=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    p = subprocess.Popen([sys.executable, "-m", "barq_inference_b200.cli", "http-server", "-m", model, "--device",
                          "cpu", "--host", "127.0.0.1", "--port", str(port), "--native-front-end"], cwd=root,
                         stdout=subprocess.PIPE, stderr=subprocess.PIPE, start_new_session=True)
    try:
        deadline = time.time() + 240
        while True:
            assert p.poll() is None, p.stderr.read().decode()[-3000:]
            try:
                if _req(port, "GET", "/health")[0] == 200:
                    break
            except OSError:
                pass
            assert time.time() < deadline, "front end did not come up"
            time.sleep(0.5)
        st, _, b = _req(port, "POST", "/v1/chat/completions",
                        {"messages": [{"role": "user", "content": "hello"}], "max_tokens": 3, "temperature": 0})
        out = json.loads(b)
        assert st == 200 and out["object"] == "chat.completion" and out["usage"]["completion_tokens"] >= 1
        assert out["model"] == "tiny.gguf"
    finally:
        os.killpg(p.pid, 15)
        p.wait(timeout=60)


def test_bench_serve_against_the_front_end(gateway):
    """The serving benchmark drives barq-http with concurrent streams and reports what it saw."""
    import asyncio

    from barq_inference_b200.server.bench_serve import run

    eng, port = gateway
    out = asyncio.run(run(f"http://127.0.0.1:{port}", n_requests=12, concurrency=4, prompt_words=3, max_tokens=4,
                          chat=True))
    assert out["completed"] == 12 and out["failed"] == 0
    assert out["output_tokens"] == 12 * 4  # the scripted engine streams 4 pieces per request
    assert 0 < out["ttft_p50_ms"] <= out["latency_p50_ms"] and out["itl_p99_ms"] >= out["itl_p50_ms"] >= 0
    assert out["request_throughput_rps"] > 0
    bad = asyncio.run(run("http://127.0.0.1:1", n_requests=2, concurrency=2, max_tokens=2))
    assert bad["completed"] == 0 and bad["failed"] == 2 and bad["errors"]


def test_several_engines_balanced_with_failover(tmp_path):
    """Two engine sockets behind one front end: concurrent requests spread over both, a dead
    engine is skipped (requests fail over), /health lists both and /metrics labels their samples."""
    import concurrent.futures as cf

    e0, e1 = FakeEngine(str(tmp_path / "a.sock")), FakeEngine(str(tmp_path / "b.sock"))
    p, port = _start(e0.path, "--socket", e1.path)
    try:
        with cf.ThreadPoolExecutor(8) as ex:
            codes = list(ex.map(lambda _: _req(port, "POST", "/v1/completions", {"prompt": "slow"})[0], range(8)))
        assert codes == [200] * 8
        assert len(e0.requests) > 0 and len(e1.requests) > 0 and len(e0.requests) + len(e1.requests) == 8
        m = _req(port, "GET", "/metrics")[2].decode()
        assert 'barq_requests_total{engine="0"} 7' in m and 'barq_requests_total{engine="1"} 7' in m
        assert m.count("# TYPE barq_requests_total counter") == 1
        e1.close()
        os.unlink(e1.path)  # engine 1 is gone: connects fail, requests go to engine 0
        n0 = len(e0.requests)
        assert all(_req(port, "POST", "/v1/completions", {"prompt": "hello"})[0] == 200 for _ in range(4))
        assert len(e0.requests) == n0 + 4
        st, _, b = _req(port, "GET", "/health")
        h = json.loads(b)
        assert st == 200 and h["status"] == "ok"
        assert [e["status"] for e in h["engines"]] == ["ok", "unreachable"]
    finally:
        p.kill()
        p.wait()
        e0.close()


def test_cli_native_front_end_with_replica_processes(tmp_path):
    """``http-server --native-front-end --dp 2``: two engine processes, each a UDS server, behind one
    barq-http; requests are served and /health lists both engines."""
    import sys

    from barq_inference_b200.cli import _engine_server_argv

    assert _engine_server_argv(["-v", "http-server", "-m", "x.gguf", "--dp", "2", "--port=9", "--host", "h",
                                "--native-front-end", "--device", "cpu"]) == ["-v", "server", "-m", "x.gguf",
                                                                            "--device", "cpu"]
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    model = str(tmp_path / "tiny.gguf")
    r = subprocess.run([sys.executable, "-m", "barq_inference_b200.cli", "make-random-gguf", "--arch", "tiny",
                        "--layers", "1", "--output", model, "--device", "cpu"], cwd=root, capture_output=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    p = subprocess.Popen([sys.executable, "-m", "barq_inference_b200.cli", "http-server", "-m", model, "--device",
                          "cpu", "--host", "127.0.0.1", "--port", str(port), "--native-front-end", "--dp", "2"],
                         cwd=root, stdout=subprocess.PIPE, stderr=subprocess.PIPE, start_new_session=True)
    try:
        deadline = time.time() + 300
        while True:
            assert p.poll() is None, p.stderr.read().decode()[-3000:]
            try:
                st, _, b = _req(port, "GET", "/health")
                if st == 200:
                    break
            except OSError:
                pass
            assert time.time() < deadline, "front end did not come up"
            time.sleep(0.5)
        h = json.loads(b)
        assert [e["status"] for e in h["engines"]] == ["ok", "ok"]
        for _ in range(4):
            st, _, b = _req(port, "POST", "/v1/completions", {"prompt": "hello", "max_tokens": 3, "temperature": 0})
            assert st == 200 and json.loads(b)["usage"]["completion_tokens"] >= 1
    finally:
        os.killpg(p.pid, 15)
        p.wait(timeout=60)


def test_api_key(tmp_path):
    eng = FakeEngine(str(tmp_path / "e.sock"))
    p, port = _start(eng.path, "--api-key", "s3cret")
    try:
        assert _req(port, "POST", "/v1/completions", {"prompt": "hello"})[0] == 401
        st, _, b = _req(port, "POST", "/v1/completions", {"prompt": "hello"}, headers={"Authorization": "Bearer nope"})
        assert st == 401 and json.loads(b)["error"]["type"] == "authentication_error"
        assert _req(port, "GET", "/v1/models", headers={"Authorization": "Bearer s3cret"})[0] == 200
        assert _req(port, "POST", "/v1/completions", {"prompt": "hello"},
                    headers={"Authorization": "Bearer s3cret"})[0] == 200
        assert _req(port, "GET", "/health")[0] == 200 and _req(port, "GET", "/metrics")[0] == 200  # stay open
        import asyncio

        from barq_inference_b200.server.bench_serve import run
        assert asyncio.run(run(f"http://127.0.0.1:{port}", n_requests=2, concurrency=2, max_tokens=2))["failed"] == 2
        assert asyncio.run(run(f"http://127.0.0.1:{port}", n_requests=2, concurrency=2, max_tokens=2,
                               api_key="s3cret"))["completed"] == 2
    finally:
        p.kill()
        p.wait()
        eng.close()


def test_remote_client_api(gateway):
    """The Client API over HTTP: generate / stream / chat / generate_batch against barq-http."""
    from barq_inference_b200.client import GenerationConfig
    from barq_inference_b200.remote import RemoteClient

    eng, port = gateway
    rc = RemoteClient(f"http://127.0.0.1:{port}", model="tiny-x")
    r = rc.generate("hello", GenerationConfig(max_tokens=4, temperature=0))
    assert r.text == "Hello world" and r.finish_reason == "length" and r.completion_tokens == 4
    assert r.prompt_tokens == 3 and r.ttft_s is not None
    assert "".join(rc.stream("hello")) == "Hello world"
    r = rc.generate("stop", GenerationConfig(stop=["<end>"]))
    assert r.text == "abc" and r.finish_reason == "stop"
    r = rc.chat([{"role": "user", "content": "hello"}], GenerationConfig(json_mode=True))
    assert r.text == "Hello world" and eng.requests[-1]["response_format"] == {"type": "json_object"}
    rs = rc.generate_batch(["hello", "utf8"])
    assert [x.text for x in rs] == ["Hello world", "é\U0001F600\"q\"\n"]
    import pytest as _pt
    with _pt.raises(RuntimeError, match="503"):
        rc.generate("queue")
