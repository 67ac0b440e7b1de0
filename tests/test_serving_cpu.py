"""Front-end contract tests on CPU: tokenizer, chat templates, grammar/JSON mode, samplers, the
OpenAI HTTP API (SSE, aliases, CORS, 429), the UDS protocol and the CLI — all on the CPU engine."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

from barq_inference_b200.engine.cpu_engine import CPUEngine
from barq_inference_b200.engine.sampling_params import SamplingParams
from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.sampling import Grammar, JSON_GBNF, schema_to_gbnf, validate_output
from barq_inference_b200.sampling.host_samplers import HostSampler, sample_chain, top_k_filter, top_p_filter
from barq_inference_b200.tokenizer import ChatTemplate, GGUFTokenizer, StreamDecoder, synthetic_tokenizer
from barq_inference_b200.tokenizer.gguf_tokenizer import bytes_to_unicode

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def tiny_engine():
    cfg = preset("tiny", n_layers=1, vocab=600, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=0)
    eng = CPUEngine(cfg, t, max_model_len=256)
    eng.tokenizer = synthetic_tokenizer(cfg.vocab)
    return eng


# ------------------------------------------------------------------ tokenizer
def test_spm_roundtrip_and_bytes():
    tok = synthetic_tokenizer(2000)
    for text in ["hello world", "the model is fast", "Zyx 123 ü€", "json: {\"a\": true}"]:
        ids = tok.encode(text, add_special=False)
        assert tok.decode(ids) == text
    ids = tok.encode("hello", add_special=True)
    assert ids[0] == tok.bos_id
    # merges prefer the highest-scoring token: "▁hello" exists as one piece
    assert tok.encode("hello", add_special=False) == [tok.vocab["▁hello"]]


def test_bpe_byte_level():
    b2u = bytes_to_unicode()
    base = [b2u[b] for b in range(256)]
    merges = ["h e", "l l", "he ll", "hell o", "Ġ w", "Ġw o", "r l", "Ġwo rl", "Ġworl d"]
    toks = base + ["he", "ll", "hell", "hello", "Ġw", "Ġwo", "rl", "Ġworl", "Ġworld", "<|end|>"]
    types = [1] * (len(toks) - 1) + [3]
    tok = GGUFTokenizer(tokens=toks, token_types=types, merges=merges, model="gpt2", add_bos=False, bos_id=None)
    ids = tok.encode("hello world<|end|>")
    assert ids == [toks.index("hello"), toks.index("Ġworld"), toks.index("<|end|>")]
    assert tok.decode(ids) == "hello world"
    assert tok.decode(tok.encode("héllo ✓")) == "héllo ✓"


def test_stream_decoder_utf8():
    tok = synthetic_tokenizer(600)
    ids = tok.encode("€", add_special=False)  # space-prefix piece + byte fallback: 3 byte tokens
    assert all(i in tok.byte_tokens.values() for i in ids[-3:])
    d = StreamDecoder(tok)
    assert [d.push(i) for i in ids][-3:] == ["", "", "€"]


def test_chat_templates():
    msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}]
    assert ChatTemplate("chatml").render(msgs).endswith("<|im_start|>assistant\n")
    l2 = ChatTemplate("llama").render(msgs)
    assert l2.startswith("[INST] <<SYS>>\nbe brief\n<</SYS>>\n\nhi [/INST]")
    l3 = ChatTemplate("llama3").render(msgs)
    assert l3.startswith("<|begin_of_text|><|start_header_id|>system<|end_header_id|>\n\nbe brief<|eot_id|>")
    src = "{% for m in messages %}<{{ m.role }}>{{ m.content }}{% endfor %}{% if add_generation_prompt %}<assistant>{% endif %}"
    assert ChatTemplate("generic", src).render(msgs) == "<system>be brief<user>hi<assistant>"
    assert ChatTemplate("generic").render([{"role": "weird", "content": "x"}]).startswith("[USER] x")


# ------------------------------------------------------------------ grammar / JSON
def test_json_grammar_and_schema():
    g = Grammar(JSON_GBNF)
    ok = g.accept_text(g.initial(), '{"a": [1, -2.5e3, true, null], "b": {"c": "x\\n"}}')
    assert Grammar.complete(ok)
    assert not g.accept_text(g.initial(), '{"a": }')
    sch = {"type": "object", "properties": {"name": {"type": "string"}, "age": {"type": "integer"},
                                            "tags": {"type": "array", "items": {"type": "string"}}},
           "required": ["name", "age"]}
    gs = Grammar(schema_to_gbnf(sch))
    assert Grammar.complete(gs.accept_text(gs.initial(), '{"name": "bo", "age": 3}'))
    assert Grammar.complete(gs.accept_text(gs.initial(), '{"name": "bo", "age": 3, "tags": ["a", "b"]}'))
    assert not gs.accept_text(gs.initial(), '{"age": 3}')
    g2 = Grammar('root ::= ("ab" | "c")+ [0-9]? # comment\n')
    assert Grammar.complete(g2.accept_text(g2.initial(), "abcab7"))
    assert not g2.accept_text(g2.initial(), "abd")


def test_json_mode_generation_is_valid(tiny_engine):
    p = SamplingParams(max_tokens=60, temperature=1.0, top_k=0, top_p=1.0, json_mode=True, seed=5)
    r = tiny_engine.generate([[1, 5, 9]], p)[0]
    text = tiny_engine.tokenizer.decode(r.tokens)
    if r.finish_reason == "stop":
        assert validate_output(text), text
    else:  # cut by max_tokens: must still be a valid JSON prefix
        g = Grammar(JSON_GBNF)
        assert g.accept_text(g.initial(), text)


# ------------------------------------------------------------------ samplers
def test_host_samplers():
    torch.manual_seed(0)
    lg = torch.randn(100)
    assert (top_k_filter(lg, 5) > -1e30).sum() == 5
    kept = top_p_filter(lg, 0.5) > -1e30
    probs = torch.softmax(lg, 0)
    assert probs[kept].sum() >= 0.5 and kept.sum() <= (probs.sort(descending=True).values.cumsum(0) < 0.5).sum() + 1
    g = torch.Generator().manual_seed(0)
    p = SamplingParams(temperature=0.0)
    assert sample_chain(lg, p, [], g) == int(lg.argmax())
    for mir in (1, 2):
        hs = HostSampler(SamplingParams(temperature=1.0, mirostat=mir, seed=1), 100)
        toks = [hs.sample(lg) for _ in range(50)]
        assert all(0 <= t < 100 for t in toks)
    hs = HostSampler(SamplingParams(temperature=1.0, typical_p=0.5, xtc_probability=1.0, xtc_threshold=0.05, seed=2), 100)
    assert 0 <= hs.sample(lg) < 100
    rep = SamplingParams(temperature=0.0, repetition_penalty=100.0)
    top = int(lg.argmax())
    assert sample_chain(lg, rep, [top], g) != top


# ------------------------------------------------------------------ HTTP API
@pytest.fixture(scope="module")
def client(tiny_engine):
    from fastapi.testclient import TestClient

    from barq_inference_b200.server.openai_api import OpenAIServer

    srv = OpenAIServer(tiny_engine, tiny_engine.tokenizer, model_id="tiny", chat_template=ChatTemplate("chatml"),
                       rate_limit_rpm=0)
    with TestClient(srv.app) as c:
        c.srv = srv
        yield c
    srv.aengine.shutdown()


def test_http_routes(client):
    r = client.get("/")
    assert r.json()["object"] == "server.info"
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    assert client.get("/health").json()["status"] == "ok"
    r = client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 5, "temperature": 0})
    j = r.json()
    assert j["object"] == "text_completion" and j["id"].startswith("cmpl-")
    assert j["usage"]["completion_tokens"] <= 5 and j["choices"][0]["finish_reason"] in ("stop", "length")
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4})
    j = r.json()
    assert j["object"] == "chat.completion" and j["choices"][0]["message"]["role"] == "assistant"
    for body in ({"input": "hey"}, {"prompt": "hey"}, {"messages": [{"role": "user", "content": "x"}]}):
        j = client.post("/v1/responses", json={**body, "max_output_tokens": 3}).json()
        assert j["object"] == "response" and j["usage"]["completion_tokens"] <= 3
    assert client.post("/v1/completions", content=b"{bad json").status_code == 400
    assert client.post("/v1/chat/completions", json={"messages": []}).status_code == 400
    assert client.get("/nope").status_code == 404
    assert client.options("/v1/completions").status_code == 204
    assert "barq_requests_total" in client.get("/metrics").text


def test_http_sse_stream(client):
    with client.stream("POST", "/v1/chat/completions",
                       json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 6, "stream": True,
                             "temperature": 0}) as r:
        events = [ln[6:] for ln in r.iter_lines() if ln.startswith("data: ")]
    assert events[-1] == "[DONE]"
    chunks = [json.loads(e) for e in events[:-1]]
    assert chunks[0]["choices"][0]["delta"] == {"role": "assistant"}
    assert all(c["object"] == "chat.completion.chunk" for c in chunks)
    assert chunks[-1]["choices"][0]["finish_reason"] in ("stop", "length")
    with client.stream("POST", "/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 3, "stream": True}) as r:
        ev = [ln[6:] for ln in r.iter_lines() if ln.startswith("data: ")]
    assert json.loads(ev[0])["object"] == "text_completion.chunk" and ev[-1] == "[DONE]"


def test_http_json_mode(client):
    j = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "json"}], "max_tokens": 40,
                                                  "response_format": {"type": "json_object"}, "temperature": 0.7,
                                                  "seed": 3}).json()
    text = j["choices"][0]["message"]["content"]
    g = Grammar(JSON_GBNF)
    assert g.accept_text(g.initial(), text)


def test_rate_limiter():
    from barq_inference_b200.server.openai_api import RateLimiter

    rl = RateLimiter(2)
    assert rl.allow("a", 0.0) and rl.allow("a", 0.0) and not rl.allow("a", 0.0)
    assert rl.allow("b", 0.0)
    assert rl.allow("a", 30.5)  # one token refilled after 30 s at 2 rpm


def test_http_429(tiny_engine):
    from fastapi.testclient import TestClient

    from barq_inference_b200.server.openai_api import OpenAIServer

    srv = OpenAIServer(tiny_engine, tiny_engine.tokenizer, rate_limit_rpm=1)
    with TestClient(srv.app) as c:
        assert c.post("/v1/completions", json={"prompt": "a", "max_tokens": 1}).status_code == 200
        r = c.post("/v1/completions", json={"prompt": "a", "max_tokens": 1})
        assert r.status_code == 429 and r.json()["error"]["type"] == "rate_limit_error"
    srv.aengine.shutdown()


# ------------------------------------------------------------------ UDS
def test_uds_protocol(tiny_engine, tmp_path):
    from barq_inference_b200.server.async_engine import AsyncEngine
    from barq_inference_b200.server.uds import UDSClient, UDSServer, recv_frame, send_frame

    path = str(tmp_path / "barq.sock")
    ae = AsyncEngine(tiny_engine)
    srv = UDSServer(ae, tiny_engine.tokenizer, path).start()
    try:
        cl = UDSClient(path)
        frames = list(cl.stream("hello", max_tokens=5, temperature=0.0, rid="r1"))
        assert frames[-1]["done"] and frames[-1]["tokens_generated"] <= 5
        assert all(f["id"] == "r1" for f in frames)
        assert all(not f["done"] for f in frames[:-1])
        # raw framing: 4-byte big-endian length + JSON
        s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        s.connect(path)
        send_frame(s, {"id": "x", "prompt": "hi", "max_tokens": 2, "temperature": 0.5})
        fr = recv_frame(s)
        assert set(fr) >= {"id", "text", "tokens_generated", "ttft_ms", "total_time_ms", "done"}
        s.close()
        cl.close()
    finally:
        srv.stop()
        ae.shutdown()


def test_native_uds_client(tiny_engine, tmp_path):
    """The C++ client against the real UDS server: a streamed request, --json prints every frame,
    --repeat summarises, a server-side error gives exit status 1, usage / connect errors give 2."""
    import shutil

    from barq_inference_b200.server.async_engine import AsyncEngine
    from barq_inference_b200.server.uds import UDSServer
    from barq_inference_b200.server.uds_native import build_client

    if shutil.which("g++") is None and shutil.which("c++") is None:
        pytest.skip("no C++ compiler")
    exe = build_client()
    path = str(tmp_path / "barq.sock")
    ae = AsyncEngine(tiny_engine)
    srv = UDSServer(ae, tiny_engine.tokenizer, path).start()
    try:
        r = subprocess.run([exe, "--socket", path, "--max-tokens", "6", "--temperature", "0", "--id", "cc",
                            'say "hi"\n\u00e9'], capture_output=True, timeout=120)
        assert r.returncode == 0, r.stderr
        assert b"[cc] tokens=" in r.stderr
        r = subprocess.run([exe, "--socket", path, "--max-tokens", "3", "--temperature", "0", "--json",
                            "--repeat", "2", "hello"], capture_output=True, timeout=120)
        assert r.returncode == 0, r.stderr
        frames = [json.loads(line) for line in r.stdout.decode().splitlines()]
        assert [f["done"] for f in frames].count(True) == 2
        assert {f["id"] for f in frames} == {"req-0", "req-1"}
        assert b"summary: requests=2" in r.stderr
        r = subprocess.run([exe, "--socket", path, "--max-tokens", "1000", "x " * 400], capture_output=True,
                           timeout=120)
        assert r.returncode == 1 and b"error=prompt exceeds max_model_len" in r.stderr
        r = subprocess.run([exe, "--socket", path, "--max-tokens", "-1", "x"], capture_output=True, timeout=60)
        assert r.returncode == 2  # usage error
        r = subprocess.run([exe, "--socket", str(tmp_path / "none.sock"), "x"], capture_output=True, timeout=60)
        assert r.returncode == 2 and b"cannot connect" in r.stderr
    finally:
        srv.stop()
        ae.shutdown()


def test_native_uds_client_decodes_frames(tmp_path):
    """Scripted server: the request the C++ client sends parses as the Python side expects, and the
    text it prints is exactly the concatenated frame texts (escapes, BMP and astral code points,
    unknown nested fields skipped)."""
    import shutil
    import threading

    from barq_inference_b200.server.uds import recv_frame, send_frame
    from barq_inference_b200.server.uds_native import build_client

    if shutil.which("g++") is None and shutil.which("c++") is None:
        pytest.skip("no C++ compiler")
    exe = build_client()
    path = str(tmp_path / "fake.sock")
    texts = ["plain ", 'quo"te\\ ', "tab\tnl\n", "\u00e9\u20ac", "\U0001F600", "/end"]
    got = {}
    lsock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    lsock.bind(path)
    lsock.listen(1)

    def serve():
        conn, _ = lsock.accept()
        got["req"] = recv_frame(conn)
        for i, t in enumerate(texts):  # json.dumps escapes non-ASCII as \uXXXX (surrogate pairs)
            send_frame(conn, {"id": got["req"]["id"], "text": t, "tokens_generated": i + 1, "ttft_ms": 5,
                              "total_time_ms": 10 + i, "done": i == len(texts) - 1, "extra": {"a": [1, "]}"]}})
        conn.close()

    th = threading.Thread(target=serve, daemon=True)
    th.start()
    prompt = 'say "hi"\n\u00e9 \U0001F600'
    r = subprocess.run([exe, "--socket", path, "--max-tokens", "7", "--temperature", "0.25", "--id", "q1", prompt],
                       capture_output=True, timeout=60)
    th.join(10)
    lsock.close()
    assert r.returncode == 0, r.stderr
    assert got["req"] == {"id": "q1", "prompt": prompt, "max_tokens": 7, "temperature": 0.25}
    assert r.stdout.decode("utf-8") == "".join(texts) + "\n"
    assert b"[q1] tokens=6 ttft_ms=5 total_ms=15" in r.stderr


# ------------------------------------------------------------------ CLI
def _cli(*args, timeout=300):
    return subprocess.run([sys.executable, "-m", "barq_inference_b200.cli", *args], cwd=ROOT, capture_output=True,
                          text=True, timeout=timeout)


def test_cli_make_info_run_convert(tmp_path):
    path = str(tmp_path / "tiny.gguf")
    r = _cli("make-random-gguf", "--arch", "tiny", "--layers", "1", "--output", path, "--device", "cpu")
    assert r.returncode == 0, r.stderr
    info = json.loads(_cli("info", "-m", path).stdout)
    assert info["architecture"] == "llama" and info["tensor_types"]["Q4_0"] > 0
    r = _cli("run", "-m", path, "--device", "cpu", "-p", "hello", "--max-tokens", "4", "--temperature", "0")
    assert r.returncode == 0, r.stderr
    out = str(tmp_path / "q8.gguf")
    r = _cli("convert", "--input", path, "--output", out, "--quantize", "q8_0", "--device", "cpu")
    assert r.returncode == 0, r.stderr
    assert json.loads(_cli("info", "-m", out).stdout)["tensor_types"].get("Q8_0", 0) > 0
    assert json.loads(_cli("metal-info").stdout)["metal"] == "unavailable"


def test_metrics_server_with_uds(tiny_engine, tmp_path):
    """Standalone metrics endpoint next to the UDS server: Prometheus text, JSON snapshot, health."""
    import json as _json
    import urllib.error
    import urllib.request

    from barq_inference_b200.server.async_engine import AsyncEngine
    from barq_inference_b200.server.metrics import InferenceMetrics
    from barq_inference_b200.server.metrics_server import MetricsServer, MetricsServerConfig
    from barq_inference_b200.server.uds import UDSClient, UDSServer

    m = InferenceMetrics()
    ae = AsyncEngine(tiny_engine)
    srv = UDSServer(ae, tiny_engine.tokenizer, str(tmp_path / "m.sock"), metrics=m).start()
    ms = MetricsServer(m, MetricsServerConfig(host="127.0.0.1", port=0), engine=tiny_engine,
                       health_fn=lambda: (ae.healthy, ae.last_error)).start()
    try:
        cl = UDSClient(str(tmp_path / "m.sock"))
        frames = list(cl.stream("hello", max_tokens=3, temperature=0.0, rid="a"))
        cl.close()
        base = f"http://127.0.0.1:{ms.port}"
        text = urllib.request.urlopen(base + "/metrics").read().decode()
        assert "barq_requests_total 1" in text and "barq_requests_successful 1" in text
        snap = _json.loads(urllib.request.urlopen(base + "/metrics.json").read())
        assert snap["tokens_generated"] == frames[-1]["tokens_generated"] and snap["requests_active"] == 0
        h = _json.loads(urllib.request.urlopen(base + "/health").read())
        assert h["status"] == "healthy" and h["metrics"]["requests_successful"] == 1
        with pytest.raises(urllib.error.HTTPError) as e:
            urllib.request.urlopen(base + "/nope")
        assert e.value.code == 404
    finally:
        ms.stop()
        srv.stop()
        ae.shutdown()


def test_prompt_tokenization_lru(tiny_engine):
    from barq_inference_b200.server.openai_api import OpenAIServer

    srv = OpenAIServer(tiny_engine, tiny_engine.tokenizer)
    try:
        srv.tok_cache_size = 2
        a = srv._encode("alpha beta")
        assert srv._encode("alpha beta") == a and srv.tok_cache_hits == 1
        srv._encode("gamma")
        srv._encode("delta")  # evicts "alpha beta" (least recently used)
        srv._encode("alpha beta")
        assert srv.tok_cache_hits == 1 and len(srv._tok_cache) == 2
    finally:
        srv.aengine.shutdown()


def test_http_n_choices_and_stream_usage(client):
    r = client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 4, "n": 3, "temperature": 0.9,
                                             "seed": 5})
    assert r.status_code == 200, r.text
    ch = r.json()["choices"]
    assert [c["index"] for c in ch] == [0, 1, 2]
    assert r.json()["usage"]["completion_tokens"] >= 3
    assert client.post("/v1/completions", json={"prompt": "hi", "n": 2, "stream": True}).status_code == 400
    with client.stream("POST", "/v1/chat/completions",
                       json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3, "stream": True,
                             "stream_options": {"include_usage": True}}) as resp:
        lines = [ln for ln in resp.iter_lines() if ln.startswith("data: ")]
    import json as _json

    last = _json.loads(lines[-2][6:])  # the chunk before [DONE]
    assert last["choices"] == [] and last["usage"]["prompt_tokens"] > 0


def test_cli_chat_and_benchmark(tmp_path):
    path = str(tmp_path / "m.gguf")
    assert _cli("make-random-gguf", "--arch", "tiny", "--layers", "1", "--output", path, "--device", "cpu").returncode == 0
    r = subprocess.run([sys.executable, "-m", "barq_inference_b200.cli", "chat", "-m", path, "--device", "cpu",
                        "--max-tokens", "4", "--temperature", "0"], cwd=ROOT, input="hello there\nand again\n/exit\n",
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.count("> ") >= 3  # two turns answered, then /exit at the third prompt
    r = _cli("benchmark", "-m", path, "--device", "cpu", "--iterations", "2", "--prompt-length", "8",
             "--gen-length", "4", "--batch", "2", "--json-out")
    assert r.returncode == 0, r.stderr[-2000:]
    summary = json.loads(r.stdout.strip().splitlines()[-1])
    assert summary["batch"] == 2 and summary["decode_tok_s"] > 0 and summary["ttft_p99_ms"] >= summary["ttft_p50_ms"]


def test_embeddings_cpu_engine_and_http(tiny_engine, client):
    import torch

    e = tiny_engine.embed([[1, 2, 3], [4, 5, 6, 7]])
    assert e.shape == (2, tiny_engine.cfg.hidden)
    assert torch.allclose(e.norm(dim=1), torch.ones(2), atol=1e-5)
    h = tiny_engine.model.forward([1, 2, 3], {}, hidden=True).mean(0)
    assert torch.allclose(e[0], h / h.norm(), atol=1e-6)
    r = client.post("/v1/embeddings", json={"input": ["hello world", "the model"]})
    assert r.status_code == 200, r.text
    d = r.json()
    assert [x["index"] for x in d["data"]] == [0, 1] and len(d["data"][0]["embedding"]) == tiny_engine.cfg.hidden
    assert d["usage"]["prompt_tokens"] > 0
    r = client.post("/v1/embeddings", json={"input": [[1, 2], [3]]})
    assert r.status_code == 200 and len(r.json()["data"]) == 2
    assert client.post("/v1/embeddings", json={"input": 5}).status_code == 400


def test_chat_tool_calls():
    from fastapi.testclient import TestClient

    from barq_inference_b200.server.openai_api import OpenAIServer

    cfg = preset("tiny", n_layers=1, vocab=600, max_ctx=2048)  # room for the tool description prompt
    eng = CPUEngine(cfg, random_tensors(cfg, POLICIES["tiny"], seed=0), max_model_len=2048)
    eng.tokenizer = synthetic_tokenizer(cfg.vocab)
    srv = OpenAIServer(eng, eng.tokenizer, chat_template=ChatTemplate("chatml"))
    client = TestClient(srv.app)
    tools = [{"type": "function", "function": {"name": "get_weather", "description": "weather for a city",
                                                "parameters": {"type": "object",
                                                               "properties": {"city": {"type": "string"}},
                                                               "required": ["city"]}}}]
    body = {"messages": [{"role": "user", "content": "weather in Paris?"}], "tools": tools, "max_tokens": 60,
            "tool_choice": {"type": "function", "function": {"name": "get_weather"}}, "temperature": 0.7, "seed": 2}
    r = client.post("/v1/chat/completions", json=body)
    assert r.status_code == 200, r.text
    ch = r.json()["choices"][0]
    if ch["finish_reason"] == "tool_calls":  # completed within max_tokens: a well-formed call
        call = ch["message"]["tool_calls"][0]
        assert call["function"]["name"] == "get_weather" and "city" in json.loads(call["function"]["arguments"])
    else:  # cut by max_tokens: still the prefix of a call
        assert ch["message"]["content"].lstrip().startswith("{")
    # the tool result goes back as a message; an assistant turn with tool_calls and no content is accepted
    body2 = {"messages": [{"role": "user", "content": "weather in Paris?"},
                          {"role": "assistant", "content": None,
                           "tool_calls": [{"id": "c1", "type": "function",
                                           "function": {"name": "get_weather", "arguments": "{\"city\": \"Paris\"}"}}]},
                          {"role": "tool", "tool_call_id": "c1", "content": "sunny"}],
             "tools": tools, "max_tokens": 5}
    assert client.post("/v1/chat/completions", json=body2).status_code == 200
    bad = dict(body, tool_choice={"type": "function", "function": {"name": "nope"}})
    assert client.post("/v1/chat/completions", json=bad).status_code == 400
    assert client.post("/v1/chat/completions", json=dict(body, stream=True)).status_code == 400
    srv.aengine.shutdown()


def test_every_subcommand_has_help():
    from barq_inference_b200.cli import build_parser

    ap = build_parser()
    sub = next(a for a in ap._actions if a.dest == "cmd")
    for name in sub.choices:
        r = _cli(name, "--help", timeout=120)
        assert r.returncode == 0 and "usage" in r.stdout.lower(), (name, r.stderr[-500:])
    assert {"run", "chat", "benchmark", "info", "convert", "server", "http-server", "metal-info",
            "wasm-info"} <= set(sub.choices)


def test_uds_disconnect_aborts_and_messages_use_the_template(tiny_engine, tmp_path):
    """A UDS client that leaves mid-stream has its request aborted in the engine (no tokens are
    generated for it afterwards); a request with chat ``messages`` is rendered with the server's
    template and its final frame carries prompt_tokens and finish_reason."""
    import time

    from barq_inference_b200.server.async_engine import AsyncEngine
    from barq_inference_b200.server.uds import UDSServer, recv_frame, send_frame

    path = str(tmp_path / "abort.sock")
    ae = AsyncEngine(tiny_engine)
    tmpl = ChatTemplate("generic")
    srv = UDSServer(ae, tiny_engine.tokenizer, path, chat_template=tmpl).start()
    try:
        msgs = [{"role": "user", "content": "hello there"}]
        s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        s.connect(path)
        send_frame(s, {"id": "m", "messages": msgs, "max_tokens": 3, "temperature": 0.0, "top_k": 1})
        frames = []
        while True:
            fr = recv_frame(s)
            frames.append(fr)
            if fr["done"]:
                break
        s.close()
        want = tiny_engine.tokenizer.encode(tmpl.render(msgs, add_generation_prompt=True), add_special=True)
        assert frames[-1]["prompt_tokens"] == len(want) and frames[-1]["finish_reason"] in ("length", "stop")
        # a long request whose client leaves after two frames
        aborted = []
        orig_abort = tiny_engine.abort

        def spy(seq, orig_abort=orig_abort):
            ok = orig_abort(seq)
            aborted.append((seq.request_id, ok, len(seq.output)))
            return ok

        tiny_engine.abort = spy
        s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        s.connect(path)
        send_frame(s, {"id": "gone", "prompt": "tell me a long story", "max_tokens": 200, "temperature": 0.0})
        recv_frame(s)
        recv_frame(s)
        s.close()
        deadline = time.time() + 30
        while time.time() < deadline and (tiny_engine.running or tiny_engine.waiting):
            time.sleep(0.05)
        assert not tiny_engine.running and not tiny_engine.waiting
        assert aborted and aborted[0][0] == "gone" and aborted[0][1] and aborted[0][2] < 200, aborted
    finally:
        tiny_engine.__dict__.pop("abort", None)
        srv.stop()
        ae.shutdown()


def test_cli_tokenize(tmp_path):
    path = str(tmp_path / "tk.gguf")
    assert _cli("make-random-gguf", "--arch", "tiny", "--layers", "1", "--output", path, "--device", "cpu").returncode == 0
    r = _cli("tokenize", "-m", path, "-p", "Hello, my name is")
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout)
    assert out["round_trip"] == "Hello, my name is" and out["n_tokens"] == len(out["ids"]) == len(out["pieces"])
    ids = _cli("tokenize", "-m", path, "-p", "Hello, my name is", "--ids-only", "--no-special").stdout.strip()
    assert [int(x) for x in ids.split(",")] == [i for i in out["ids"] if i != 1]


def test_http_logprobs(client, tiny_engine):
    """logprobs / top_logprobs: one entry per generated token with the model's log-softmax; greedy
    picks the most likely token, so it equals the first alternative; completions carry tokens,
    token_logprobs, top_logprobs and text offsets, also in SSE chunks."""
    import math

    body = {"messages": [{"role": "user", "content": "hello"}], "max_tokens": 6, "temperature": 0,
            "logprobs": True, "top_logprobs": 3}
    out = client.post("/v1/chat/completions", json=body).json()
    ch = out["choices"][0]
    ents = ch["logprobs"]["content"]
    assert len(ents) == out["usage"]["completion_tokens"] > 0
    for e in ents:
        assert e["logprob"] <= 0 and len(e["top_logprobs"]) == 3
        alts = [a["logprob"] for a in e["top_logprobs"]]
        assert alts == sorted(alts, reverse=True)
        assert math.isclose(e["logprob"], alts[0], abs_tol=1e-5)  # greedy = the most likely token
        assert e["token"] == e["top_logprobs"][0]["token"] and bytes(e["bytes"]).decode("utf-8", "replace") == e["token"]
    # without logprobs the field is null
    assert client.post("/v1/chat/completions", json={**body, "logprobs": False}).json()["choices"][0]["logprobs"] is None
    r = client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 5, "temperature": 0.7, "seed": 3,
                                             "logprobs": 2}).json()
    lp = r["choices"][0]["logprobs"]
    n = r["usage"]["completion_tokens"]
    assert len(lp["tokens"]) == len(lp["token_logprobs"]) == len(lp["top_logprobs"]) == len(lp["text_offset"]) == n
    assert all(len(t) <= 2 for t in lp["top_logprobs"]) and lp["text_offset"] == sorted(lp["text_offset"])
    assert "".join(lp["tokens"]) == r["choices"][0]["text"]
    # streamed: every chunk carries the entries of its own tokens
    with client.stream("POST", "/v1/chat/completions", json={**body, "stream": True}) as resp:
        evs = [json.loads(line[6:]) for line in resp.iter_lines() if line.startswith("data: ") and "[DONE]" not in line]
    streamed = [e for ev in evs for e in (ev["choices"][0].get("logprobs") or {}).get("content", [])]
    assert [e["token"] for e in streamed] == [e["token"] for e in ents]
    assert client.post("/v1/completions", json={"prompt": "x", "logprobs": 21}).status_code == 400


def test_http_stop_string_is_never_streamed(client, tiny_engine):
    """A stop string split across streamed pieces is held back: no chunk contains any part of it."""
    r = client.post("/v1/completions", json={"prompt": "hello", "max_tokens": 24, "temperature": 0}).json()
    text = r["choices"][0]["text"]
    if len(text) < 6:
        pytest.skip("greedy continuation too short for a split stop string")
    stop = text[3:6]
    with client.stream("POST", "/v1/completions",
                       json={"prompt": "hello", "max_tokens": 24, "temperature": 0, "stop": [stop], "stream": True}) as resp:
        evs = [json.loads(line[6:]) for line in resp.iter_lines() if line.startswith("data: ") and "[DONE]" not in line]
    pieces = [e["choices"][0]["text"] for e in evs]
    assert "".join(pieces) == text[:text.find(stop)]
    assert evs[-1]["choices"][0]["finish_reason"] == "stop"


def test_native_uds_client_chat_mode(tmp_path):
    """barq-uds --chat: one user turn per stdin line, the whole history (system, user, assistant
    replies) sent as OpenAI messages; a failed turn is dropped from the history."""
    import shutil
    import threading

    from barq_inference_b200.server.uds import recv_frame, send_frame
    from barq_inference_b200.server.uds_native import build_client

    if shutil.which("g++") is None and shutil.which("c++") is None:
        pytest.skip("no C++ compiler")
    exe = build_client()
    path = str(tmp_path / "chat.sock")
    seen = []
    lsock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
    lsock.bind(path)
    lsock.listen(1)

    def serve():
        conn, _ = lsock.accept()
        while True:
            req = recv_frame(conn)
            if req is None:
                break
            seen.append(req)
            last = req["messages"][-1]["content"]
            if last == "fail":
                send_frame(conn, {"id": req["id"], "text": "", "done": True, "error": "queue full"})
                continue
            for i, t in enumerate(["re: ", last]):
                send_frame(conn, {"id": req["id"], "text": t, "tokens_generated": i + 1, "done": False})
            send_frame(conn, {"id": req["id"], "text": "", "tokens_generated": 2, "done": True})
        conn.close()

    th = threading.Thread(target=serve, daemon=True)
    th.start()
    r = subprocess.run([exe, "--socket", path, "--chat", "--system", "be brief", "--max-tokens", "9"],
                       input="hello\nfail\nagain é\n/exit\nignored\n".encode(), capture_output=True, timeout=60)
    th.join(10)
    lsock.close()
    assert r.returncode == 1, r.stderr  # one turn failed
    assert r.stdout.decode() == "re: hello\n\nre: again é\n"
    assert [q["messages"] for q in seen] == [
        [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hello"}],
        [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hello"},
         {"role": "assistant", "content": "re: hello"}, {"role": "user", "content": "fail"}],
        [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hello"},
         {"role": "assistant", "content": "re: hello"}, {"role": "user", "content": "again é"}]]
    assert all(q["max_tokens"] == 9 for q in seen)


def test_uds_prompt_cache(tiny_engine, tmp_path):
    """Repeated prompt texts (and rendered chat prompts) skip the tokenizer on the UDS server."""
    from barq_inference_b200.server.async_engine import AsyncEngine
    from barq_inference_b200.server.uds import UDSClient, UDSServer

    path = str(tmp_path / "pc.sock")
    ae = AsyncEngine(tiny_engine)
    srv = UDSServer(ae, tiny_engine.tokenizer, path).start()
    try:
        cl = UDSClient(path)
        a = [f["text"] for f in cl.stream("same words again", max_tokens=3, temperature=0.0)]
        b = [f["text"] for f in cl.stream("same words again", max_tokens=3, temperature=0.0)]
        cl.close()
        assert a and b and srv.tok_cache_hits == 1  # (the texts may differ: near-tied random logits)
        assert srv._encode("same words again") == tiny_engine.tokenizer.encode("same words again")
    finally:
        srv.stop()
        ae.shutdown()


def test_http_api_key(tiny_engine):
    from fastapi.testclient import TestClient

    from barq_inference_b200.server.openai_api import OpenAIServer

    srv = OpenAIServer(tiny_engine, tiny_engine.tokenizer, model_id="tiny", rate_limit_rpm=0, api_key="k1")
    with TestClient(srv.app) as c:
        body = {"prompt": "hello", "max_tokens": 2}
        r = c.post("/v1/completions", json=body)
        assert r.status_code == 401 and r.json()["error"]["type"] == "authentication_error"
        assert c.post("/v1/completions", json=body, headers={"Authorization": "Bearer k2"}).status_code == 401
        assert c.post("/v1/completions", json=body, headers={"Authorization": "Bearer k1"}).status_code == 200
        assert c.get("/health").status_code == 200
    srv.aengine.shutdown()


def test_uds_health_and_metrics_queries(tiny_engine, tmp_path):
    import shutil

    from barq_inference_b200.server.async_engine import AsyncEngine
    from barq_inference_b200.server.uds import UDSClient, UDSServer
    from barq_inference_b200.server.uds_native import build_client

    path = str(tmp_path / "hm.sock")
    ae = AsyncEngine(tiny_engine)
    srv = UDSServer(ae, tiny_engine.tokenizer, path).start()
    try:
        cl = UDSClient(path)
        list(cl.stream("hi", max_tokens=2, temperature=0.0))
        h = cl.query("health")
        assert h["healthy"] is True and h["done"] is True
        m = cl.query("metrics")["prometheus"]
        assert "barq_requests_total 1" in m
        cl.close()
        if shutil.which("g++") or shutil.which("c++"):
            exe = build_client()
            r = subprocess.run([exe, "--socket", path, "--health"], capture_output=True, timeout=60)
            assert r.returncode == 0 and json.loads(r.stdout)["healthy"] is True
            r = subprocess.run([exe, "--socket", path, "--metrics"], capture_output=True, timeout=60)
            assert r.returncode == 0 and b"barq_requests_total" in r.stdout
    finally:
        srv.stop()
        ae.shutdown()


def test_http_tokenize_detokenize(client, tiny_engine):
    tok = tiny_engine.tokenizer
    r = client.post("/tokenize", json={"content": "hello there"}).json()
    assert r["tokens"] == tok.encode("hello there", add_special=False)
    assert client.post("/detokenize", json={"tokens": r["tokens"]}).json()["content"] == tok.decode(r["tokens"])
    assert client.post("/tokenize", json={"content": 3}).status_code == 400
    assert client.post("/detokenize", json={"tokens": [-1]}).status_code == 400


def test_http_retrieve_model(client):
    assert client.get("/v1/models/tiny").json()["id"] == "tiny"
    assert client.get("/v1/models/other").status_code == 404


def test_uds_socket_is_owner_only(tiny_engine, tmp_path, monkeypatch):
    import stat

    from barq_inference_b200.server.async_engine import AsyncEngine
    from barq_inference_b200.server.uds import UDSServer

    ae = AsyncEngine(tiny_engine)
    path = str(tmp_path / "perm.sock")
    srv = UDSServer(ae, tiny_engine.tokenizer, path).start()
    try:
        assert stat.S_IMODE(os.stat(path).st_mode) == 0o600
    finally:
        srv.stop()
    monkeypatch.setenv("BARQ_SOCKET_MODE", "660")
    srv = UDSServer(ae, tiny_engine.tokenizer, path).start()
    try:
        assert stat.S_IMODE(os.stat(path).st_mode) == 0o660
    finally:
        srv.stop()
        ae.shutdown()


def test_http_batch_of_prompts(client):
    r = client.post("/v1/completions", json={"prompt": ["one", "two words", "three"], "max_tokens": 2,
                                             "temperature": 0, "n": 2}).json()
    assert [c["index"] for c in r["choices"]] == list(range(6))
    assert r["usage"]["completion_tokens"] > 0
    r2 = client.post("/v1/completions", json={"prompt": [[1, 2, 3], [4, 5]], "max_tokens": 1}).json()
    assert len(r2["choices"]) == 2 and r2["usage"]["prompt_tokens"] == 5
    assert client.post("/v1/completions", json={"prompt": ["a", "b"], "stream": True}).status_code == 400
