"""Data-parallel replicas on CPU: replica processes built by a factory, least-outstanding-work routing,
prefix affinity, a replica that dies, and the OpenAI server over the replica front end."""
import pytest

from barq_inference_b200.engine.cpu_engine import CPUEngine
from barq_inference_b200.engine.sampling_params import SamplingParams
from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.parallel.dp import DataParallelEngine, PresetEngineFactory
from barq_inference_b200.tokenizer.gguf_tokenizer import synthetic_tokenizer

OVR = dict(n_layers=1, vocab=600, max_ctx=256)


def _factory():
    return PresetEngineFactory("tiny", OVR, seed=0, engine_kw={"max_model_len": 256})


@pytest.fixture(scope="module")
def dp():
    cfg = preset("tiny", **OVR)
    front = DataParallelEngine(_factory(), ["cpu", "cpu"], cfg=cfg, tokenizer=synthetic_tokenizer(cfg.vocab),
                               affinity_tokens=8, affinity_slack=10_000, start_timeout=300)
    yield front
    front.shutdown()


def test_dp_greedy_matches_single_engine(dp):
    cfg = preset("tiny", **OVR)
    single = CPUEngine(cfg, random_tensors(cfg, POLICIES["tiny"], seed=0), max_model_len=256)
    prompts = [[1 + i, 7, 9 + 3 * i, 22, 5 + i] for i in range(6)]
    p = SamplingParams.greedy_params(max_tokens=6)
    want = [r.tokens for r in single.generate(prompts, p)]
    got = dp.generate(prompts, p)
    assert got == want
    info = dp.replica_info()
    assert all(r["alive"] for r in info)
    assert all(r["served"] > 0 for r in info), info  # both replicas took work
    assert all(r["load"] == 0 for r in info), info  # every finished request returned its cost


def test_dp_least_loaded_and_affinity():
    """Routing decisions on a front end with no processes: lowest outstanding tokens wins; a prompt
    whose prefix was served before returns to that replica while within the slack."""
    from barq_inference_b200.parallel.dp import ReplicaState

    fe = DataParallelEngine.__new__(DataParallelEngine)
    fe.replicas = [ReplicaState(0, "cpu", alive=True, load=500), ReplicaState(1, "cpu", alive=True, load=100),
                   ReplicaState(2, "cpu", alive=False, load=0)]
    fe.affinity_tokens, fe.affinity_slack, fe._affinity, fe.last_error = 4, 450, {}, None
    assert fe._pick([1, 2, 3], 10) == 1  # short prompt: no affinity, least loaded live replica
    fe._affinity[(9, 9, 9, 9)] = 0
    assert fe._pick([9, 9, 9, 9, 5], 10) == 0  # 500 <= 100 + 450: stays on the replica holding the prefix
    fe.replicas[0].load = 600
    assert fe._pick([9, 9, 9, 9, 5], 10) == 1  # too far behind: moves, and the prefix now maps to 1
    assert fe._affinity[(9, 9, 9, 9)] == 1
    for r in fe.replicas:
        r.alive = False
    with pytest.raises(RuntimeError):
        fe._pick([1], 1)


def test_dp_openai_server_over_replicas(dp):
    from fastapi.testclient import TestClient

    from barq_inference_b200.server.openai_api import OpenAIServer
    from barq_inference_b200.tokenizer import ChatTemplate

    srv = OpenAIServer(dp, dp.tokenizer, model_id="tiny-dp", chat_template=ChatTemplate("chatml"), aengine=dp)
    c = TestClient(srv.app)
    r = c.post("/v1/completions", json={"prompt": "hello world", "max_tokens": 5, "temperature": 0})
    assert r.status_code == 200, r.text
    assert r.json()["usage"]["completion_tokens"] >= 1
    h = c.get("/health")
    assert h.status_code == 200 and h.json()["status"] == "ok"
    # logprobs recorded on the replica reach the server: one entry per token, greedy = top alternative
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 4,
                                             "temperature": 0, "logprobs": True, "top_logprobs": 2}).json()
    ents = r["choices"][0]["logprobs"]["content"]
    assert len(ents) == r["usage"]["completion_tokens"] >= 1
    assert all(abs(e["logprob"] - e["top_logprobs"][0]["logprob"]) < 1e-5 for e in ents)


def test_dp_replica_death_fails_its_requests_only():
    cfg = preset("tiny", **OVR)
    front = DataParallelEngine(_factory(), ["cpu", "cpu"], cfg=cfg, affinity_tokens=0, start_timeout=300)
    try:
        victim = front.replicas[0]
        victim.proc.kill()
        victim.proc.join(timeout=30)
        p = SamplingParams.greedy_params(max_tokens=4)
        import time

        deadline = time.monotonic() + 30
        while victim.alive and time.monotonic() < deadline:
            time.sleep(0.05)
        assert not victim.alive and "exited" in (victim.error or "")
        assert front.healthy and front.n_alive == 1
        outs = front.generate([[3, 4, 5], [6, 7, 8]], p)  # all routed to the survivor
        assert [len(o) for o in outs] == [4, 4]
        assert front.replicas[1].served == 2
    finally:
        front.shutdown()


def test_cli_dp_front_from_gguf(tmp_path):
    """``--dp 2`` as the servers build it: replicas load the GGUF file themselves (GGUFEngineFactory)."""
    from barq_inference_b200.cli import _dp_front, build_parser, main

    path = str(tmp_path / "m.gguf")
    assert main(["make-random-gguf", "--arch", "tiny", "--layers", "1", "--output", path, "--device", "cpu"]) == 0
    args = build_parser().parse_args(["server", "-m", path, "--device", "cpu", "--dp", "2", "--context-size", "128"])
    front, tok, _ = _dp_front(args)
    try:
        assert front.n_alive == 2
        outs = front.generate([[1, 2, 3], [4, 5, 6], [7, 8, 9]], SamplingParams.greedy_params(max_tokens=3))
        assert [len(o) for o in outs] == [3, 3, 3]
    finally:
        front.shutdown()


def test_dp_stream_closed_early_cancels_on_the_replica(dp):
    import asyncio
    import time

    async def two():
        agen = dp.stream([1, 2, 3, 4], SamplingParams(max_tokens=200, temperature=0.0, ignore_eos=True))
        got = [await agen.__anext__(), await agen.__anext__()]
        await agen.aclose()
        return got

    got = asyncio.run(two())
    assert all(g.token is not None for g in got)
    deadline = time.monotonic() + 30
    while any(r["load"] for r in dp.replica_info()) and time.monotonic() < deadline:
        time.sleep(0.05)
    assert all(r["load"] == 0 for r in dp.replica_info())
    assert not dp._reqs  # nothing left in flight


def test_dp_replica_killed_mid_stream_does_not_silence_the_survivor():
    """A replica killed while it streams tokens (possibly in the middle of a message to the front
    end) fails only its own requests: each replica writes to its own pipe, so the survivor's
    stream keeps arriving and finishes."""
    import queue as q
    import time

    cfg = preset("tiny", **OVR)
    front = DataParallelEngine(_factory(), ["cpu", "cpu"], cfg=cfg, affinity_tokens=0, start_timeout=300)
    try:
        p = SamplingParams.greedy_params(max_tokens=40)
        p.ignore_eos = True
        reqs = [front._submit([3 + i, 4, 5], p, f"r{i}", sink=q.Queue()) for i in range(4)]
        by_rep = {}
        for r in reqs:
            by_rep.setdefault(r.replica, []).append(r)
        assert set(by_rep) == {0, 1}, "both replicas took requests"
        victim = front.replicas[0]
        first = by_rep[0][0].sink.get(timeout=300)  # replica 0 is streaming
        assert first.token is not None
        victim.proc.kill()
        for r in by_rep[1]:  # the survivor's requests run to their end
            n, deadline = 0, time.monotonic() + 300  # generous: CPU tests may share the cores
            while True:
                item = r.sink.get(timeout=max(1.0, deadline - time.monotonic()))
                if item.token is None:
                    break
                n += 1
            assert item.finish_reason == "length" and n == 40
        for r in by_rep[0]:  # the victim's requests end: with an error, unless they finished first
            while True:
                item = r.sink.get(timeout=300)
                if item.token is None:
                    break
            assert item.finish_reason.startswith("error") or item.finish_reason == "length"
        assert front.n_alive == 1
    finally:
        front.shutdown()
