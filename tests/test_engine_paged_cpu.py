"""The CUDA engine's host logic end to end on CPU: ``Engine`` (scheduler, chunked prefill, paged-KV
slots and block tables, preemption, prefix cache, sliding-window page freeing, sampling plumbing)
driving a paged fp32 runner that stores K/V at exactly the slots the engine hands it and attends
through the block tables.  Its greedy tokens must follow the contiguous fp32 reference forward: a
wrong slot, position or block table shows up as different logits."""
import dataclasses

import pytest
import torch

import barq_inference_b200.engine.engine as engine_mod
from barq_inference_b200.engine.engine import Engine, EngineConfig
from barq_inference_b200.engine.sampling_params import SamplingParams
from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.models.reference import ReferenceModel, rms_norm
from barq_inference_b200.models.rope import apply_rope_ref


class PagedRefRunner:
    """fp32 forward over a paged K/V store, following the reference model's math."""

    def __init__(self, cfg, tensors):
        self.cfg = cfg
        self.ref = ReferenceModel(cfg, tensors)
        self.w = self.ref.w

    def kv_bytes_per_block(self, block_size=16):
        c = self.cfg
        return c.n_layers * 2 * c.n_kv_heads * block_size * c.head_dim * 4

    def allocate_kv(self, num_blocks, block_size=16):
        c = self.cfg
        self.bs = block_size
        self.kc = torch.full((c.n_layers, num_blocks * block_size, c.n_kv_heads, c.head_dim), float("nan"))
        self.vc = torch.full_like(self.kc, float("nan"))  # unwritten slots are NaN: reading one poisons logits
        # the device runner's page layout [blocks, kv heads, block_size, head_dim], as strided views
        pages = lambda t: t.view(num_blocks, block_size, c.n_kv_heads, c.head_dim).permute(0, 2, 1, 3)  # noqa: E731
        self.kv = [(pages(self.kc[i]), pages(self.vc[i])) for i in range(c.n_layers)]
        return self.kv

    def forward(self, inp):
        cfg, w, ref = self.cfg, self.w, self.ref
        ids = inp.ids.long()
        pos = inp.pos.long()
        slots = inp.slots.long()
        T = ids.numel()
        S = inp.seq_lens.numel()
        if inp.decode:
            rows = [(s, s + 1) for s in range(S)]
        else:
            qs = inp.q_start.tolist()
            rows = [(qs[s], qs[s + 1]) for s in range(S)]
        x = w["token_embd.weight"][ids].clone()
        if inp.embed_rows is not None and inp.embed_rows.numel():  # multimodal rows
            x[inp.embed_rows.long()] = inp.embed_vals.float()
        cos, sin = ref.cos[pos], ref.sin[pos]
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            h = rms_norm(x, w[p + "attn_norm.weight"], cfg.rms_eps)
            q = (h @ w[p + "attn_q.weight"].T).view(T, cfg.n_heads, cfg.head_dim)
            k = (h @ w[p + "attn_k.weight"].T).view(T, cfg.n_kv_heads, cfg.head_dim)
            v = (h @ w[p + "attn_v.weight"].T).view(T, cfg.n_kv_heads, cfg.head_dim)
            r = cfg.rot_dim
            q = torch.cat([apply_rope_ref(q[..., :r], cos, sin, cfg.rope_neox), q[..., r:]], -1)
            k = torch.cat([apply_rope_ref(k[..., :r], cos, sin, cfg.rope_neox), k[..., r:]], -1)
            self.kc[i, slots] = k
            self.vc[i, slots] = v
            o = torch.empty(T, cfg.n_heads, cfg.head_dim)
            for s, (a, b) in enumerate(rows):
                L = int(inp.seq_lens[s])
                kp = torch.arange(L)
                if cfg.sliding_window:  # only positions some query of the chunk can attend to are read
                    kp = kp[kp >= int(pos[a]) - cfg.sliding_window + 1]
                bt = inp.block_tables[s].long()
                ks = bt[kp // self.bs] * self.bs + kp % self.bs
                kk, vv = self.kc[i, ks], self.vc[i, ks]
                qpos = pos[a:b][:, None]
                rep = cfg.n_heads // cfg.n_kv_heads
                kk, vv = kk.repeat_interleave(rep, 1), vv.repeat_interleave(rep, 1)
                sc = torch.einsum("thd,shd->hts", q[a:b], kk) * ref.scale
                mask = kp[None, :] > qpos
                if cfg.sliding_window:
                    mask |= kp[None, :] <= qpos - cfg.sliding_window
                sc = sc.masked_fill(mask[None], float("-inf"))
                o[a:b] = torch.einsum("hts,shd->thd", torch.softmax(sc, -1), vv)
            x = x + o.reshape(T, -1) @ w[p + "attn_output.weight"].T
            h = rms_norm(x, w[p + "ffn_norm.weight"], cfg.rms_eps)
            x = x + (ref._moe(h, p) if cfg.layer_is_moe(i) else ref._ffn(h, p))
        xl = x[inp.last_idx.long()] if not inp.decode else x
        xl = rms_norm(xl, w["output_norm.weight"], cfg.rms_eps)
        return xl @ w.get("output.weight", w["token_embd.weight"]).T


def _greedy_sample(logits, temp, topk, topp, minp, seeds, steps, allow_mask=None, penalties=None, history=None,
                   want_logprob=False):
    lg = logits.float().clone()
    if allow_mask is not None:
        bits = ((allow_mask.view(torch.int32).long()[:, :, None] >> torch.arange(32)) & 1).reshape(lg.shape[0], -1)
        lg = lg.masked_fill(bits[:, : lg.shape[1]] == 0, float("-inf"))
    return lg.argmax(-1).to(torch.int32), None


@pytest.fixture(autouse=True)
def _cpu_sampler(monkeypatch):
    monkeypatch.setattr(engine_mod.ops, "sample", _greedy_sample)


def _follows_reference(ref: ReferenceModel, prompt, tokens, tol=1e-3):
    """True if ``tokens`` is the reference's greedy continuation, allowing a switch only where the
    reference's top two logits are within ``tol`` (a near-tie that rounding may flip)."""
    cache: dict = {}
    logits = ref.forward(prompt, cache)[-1]
    for t in tokens:
        best = int(logits.argmax())
        if t != best:
            return bool(logits[best] - logits[t] < tol)
        logits = ref.forward([t], cache)[-1]
    return True


def _engine(cfg, tensors, **kw):
    ec = EngineConfig(device="cpu", cuda_graphs=False, max_model_len=256, **kw)
    return Engine(cfg, tensors, ec, runner=PagedRefRunner(cfg, tensors))


def _prompts(cfg, n, seed, lo=5, hi=70, shared=0):
    g = torch.Generator().manual_seed(seed)
    base = torch.randint(0, cfg.vocab, (shared,), generator=g).tolist()
    return [base + torch.randint(0, cfg.vocab, (int(torch.randint(lo, hi, (1,), generator=g)),), generator=g).tolist()
            for _ in range(n)]


def test_continuous_batching_chunked_prefill_matches_reference():
    cfg = preset("tiny", n_layers=2, vocab=500, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=0)
    ref = ReferenceModel(cfg, t)
    eng = _engine(cfg, t, num_blocks=64, max_num_batched_tokens=24, max_num_seqs=3)
    prompts = _prompts(cfg, 5, 1)
    res = eng.generate(prompts, SamplingParams.greedy_params(max_tokens=12))
    for p, r in zip(prompts, res):
        assert len(r.tokens) == 12 and _follows_reference(ref, p, r.tokens)


def test_preemption_under_a_small_pool_matches_reference():
    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=2)
    ref = ReferenceModel(cfg, t)
    eng = _engine(cfg, t, num_blocks=12, max_num_batched_tokens=64, max_num_seqs=4)
    prompts = _prompts(cfg, 4, 3, lo=30, hi=50)
    res = eng.generate(prompts, SamplingParams.greedy_params(max_tokens=30))
    assert eng.sched.n_preemptions > 0
    for p, r in zip(prompts, res):
        assert len(r.tokens) == 30 and _follows_reference(ref, p, r.tokens)


def test_host_sampled_rows_in_a_mixed_batch_match_reference():
    """Sequences sampled on the host (Mirostat v2 with a tiny target surprise keeps only the most
    likely token) share decode batches with device-sampled greedy ones: each host row must get its
    own sequence's logits, so every sequence follows the reference's greedy continuation."""
    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=6)
    ref = ReferenceModel(cfg, t)
    eng = _engine(cfg, t, num_blocks=64, max_num_batched_tokens=128, max_num_seqs=4)
    prompts = _prompts(cfg, 4, 7)
    params = [SamplingParams.greedy_params(max_tokens=10),
              SamplingParams(temperature=1.0, mirostat=2, mirostat_tau=0.01, max_tokens=10, seed=1),
              SamplingParams.greedy_params(max_tokens=10),
              SamplingParams(temperature=1.0, mirostat=2, mirostat_tau=0.01, max_tokens=10, seed=2)]
    res = eng.generate(prompts, params)
    for p, r in zip(prompts, res):
        assert len(r.tokens) == 10 and _follows_reference(ref, p, r.tokens)


def test_prefix_cache_reuse_matches_reference():
    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=4)
    ref = ReferenceModel(cfg, t)
    eng = _engine(cfg, t, num_blocks=64, max_num_batched_tokens=128, max_num_seqs=4, prefix_caching=True)
    prompts = _prompts(cfg, 4, 5, lo=3, hi=10, shared=40)
    first = eng.generate(prompts[:1], SamplingParams.greedy_params(max_tokens=6))
    rest = eng.generate(prompts[1:], SamplingParams.greedy_params(max_tokens=6))
    assert eng.prefix_cache.hits >= 3
    for p, r in zip(prompts, first + rest):
        assert _follows_reference(ref, p, r.tokens)


def test_sliding_window_page_freeing_matches_reference():
    cfg = dataclasses.replace(preset("tiny", n_layers=1, vocab=400, max_ctx=256), sliding_window=24)
    t = random_tensors(cfg, POLICIES["tiny"], seed=6)
    ref = ReferenceModel(cfg, t)
    eng = _engine(cfg, t, num_blocks=20, max_num_batched_tokens=16, max_num_seqs=2)
    prompts = _prompts(cfg, 2, 7, lo=40, hi=60)
    res = eng.generate(prompts, SamplingParams.greedy_params(max_tokens=60))
    assert eng.sched.n_window_freed > 0
    for p, r in zip(prompts, res):
        assert _follows_reference(ref, p, r.tokens)


@pytest.mark.parametrize("seed,prefix,window", [(0, False, 0), (1, True, 0), (2, False, 24), (3, True, 0)])
def test_random_arrivals_aborts_and_preemption_follow_reference(seed, prefix, window):
    """Randomized serving on a small pool: requests arrive between steps, some clients go away,
    prompts share prefixes, the pool forces preemption (and window release).  Every request that
    finishes by length must be the reference's greedy continuation; aborted ones free their pages."""
    import random

    rng = random.Random(seed)
    cfg = dataclasses.replace(preset("tiny", n_layers=1, vocab=400, max_ctx=256), sliding_window=window)
    t = random_tensors(cfg, POLICIES["tiny"], seed=20 + seed)
    ref = ReferenceModel(cfg, t)
    eng = _engine(cfg, t, num_blocks=rng.choice([14, 20]), max_num_batched_tokens=rng.choice([16, 40]),
                  max_num_seqs=rng.choice([3, 4]), prefix_caching=prefix)
    shared = torch.randint(0, cfg.vocab, (32,), generator=torch.Generator().manual_seed(seed)).tolist()
    pending = []
    for i in range(10):
        base = shared[: rng.choice([0, 16, 32])] if prefix else []
        prompt = base + [rng.randrange(cfg.vocab) for _ in range(rng.randint(3, 40))]
        pending.append((prompt, SamplingParams.greedy_params(max_tokens=rng.randint(4, 24))))
    live, done, aborted = [], [], []
    steps = 0
    while pending or eng.has_work():
        if pending and (rng.random() < 0.5 or not eng.has_work()):
            p, sp = pending.pop(0)
            live.append(eng.add_request(p, sp))
        if live and rng.random() < 0.06:
            s = live.pop(rng.randrange(len(live)))
            if eng.abort(s):
                aborted.append(s)
        for s in eng.step():
            done.append(s)
        steps += 1
        assert steps < 5000
    finished = [s for s in done if s.finish_reason == "length"]
    assert finished
    for s in finished:
        assert len(s.output) == s.params.max_tokens and _follows_reference(ref, s.prompt, s.output)
    assert all(not s.block_table for s in aborted + done)
    held = eng.prefix_cache.n_blocks if eng.prefix_cache is not None else 0
    assert eng.blocks.n_used == 1 + held  # the dummy page plus what the prefix cache keeps
    if prefix:  # these workloads overfill the pool
        assert eng.sched.n_preemptions > 0 and eng.prefix_cache.hits > 0
    if window:
        assert eng.sched.n_window_freed > 0


def test_kv_session_export_import_through_the_engine(tmp_path):
    from barq_inference_b200.engine.session import export_session, import_session

    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=8)
    ref = ReferenceModel(cfg, t)
    system = _prompts(cfg, 1, 9, lo=40, hi=41)[0]
    a = _engine(cfg, t, num_blocks=64, max_num_batched_tokens=128, prefix_caching=True)
    path = str(tmp_path / "s.pt")
    st = export_session(a, system, path)
    assert st["tokens"].numel() == 32  # whole pages of the cached prefix
    b = _engine(cfg, t, num_blocks=64, max_num_batched_tokens=128, prefix_caching=True)
    assert import_session(b, path) == 32
    prompt = system + [7, 8, 9]
    r = b.generate([prompt], SamplingParams.greedy_params(max_tokens=8))[0]
    assert b.prefix_cache.hits >= 1 and b.timings["prefill_tokens"] == len(prompt) - 32
    assert _follows_reference(ref, prompt, r.tokens)


def test_multimodal_embedding_rows_through_the_engine():
    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=10)
    ref = ReferenceModel(cfg, t)
    prompt = _prompts(cfg, 1, 11, lo=30, hi=31)[0]
    rows = torch.randn(6, cfg.hidden, generator=torch.Generator().manual_seed(12)) * 0.5
    eng = _engine(cfg, t, num_blocks=64, max_num_batched_tokens=16)  # the image rows straddle two chunks
    seq = eng.add_request(prompt, SamplingParams.greedy_params(max_tokens=6), embeds=(12, rows))
    while eng.has_work():
        eng.step()
    cache: dict = {}
    logits = ref.forward(prompt, cache, embeds=(12, rows))[-1]
    for tok in seq.output:
        best = int(logits.argmax())
        assert tok == best or logits[best] - logits[tok] < 1e-3
        if tok != best:
            break
        logits = ref.forward([tok], cache)[-1]


def test_json_mode_mask_plumbing_through_the_engine():
    import json as _json

    from barq_inference_b200.tokenizer.gguf_tokenizer import synthetic_tokenizer

    cfg = preset("tiny", n_layers=1, vocab=600, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=12)
    eng = _engine(cfg, t, num_blocks=64, max_num_batched_tokens=64)
    eng.tokenizer = synthetic_tokenizer(cfg.vocab)
    r = eng.generate([[1, 5, 9]], SamplingParams(max_tokens=64, temperature=0.0, json_mode=True))[0]
    text = eng.tokenizer.decode([x for x in r.tokens if x not in cfg.eos_ids])
    if r.finish_reason == "stop":
        _json.loads(text)
    else:  # ran out of tokens: still a valid JSON prefix under the grammar
        assert text.lstrip().startswith("{")


@pytest.mark.parametrize("same_draft", [True, False])
def test_speculative_greedy_follows_target_reference(same_draft):
    """Speculative decoding through the real engines' paged state: greedy output is the target's
    greedy continuation whatever the draft; an identical draft is (almost) always accepted."""
    from barq_inference_b200.engine.speculative import SpeculativeConfig, SpeculativeDecoder

    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=13)
    d = t if same_draft else random_tensors(cfg, POLICIES["tiny"], seed=14)
    ref = ReferenceModel(cfg, t)
    target = _engine(cfg, t, num_blocks=64)
    draft = _engine(cfg, d, num_blocks=64)
    prompt = _prompts(cfg, 1, 15, lo=20, hi=21)[0]
    res = SpeculativeDecoder(target, draft, SpeculativeConfig(4)).generate(
        prompt, SamplingParams.greedy_params(max_tokens=20))
    assert len(res.tokens) == 20 and _follows_reference(ref, prompt, res.tokens)
    if same_draft:
        assert res.acceptance_rate > 0.9
    assert target.blocks.n_used == 1 and draft.blocks.n_used == 1  # pages released (dummy page only)


def test_openai_server_over_the_engine():
    """The HTTP server with the CUDA engine's host side (AsyncEngine thread, KV gauges, health)."""
    from fastapi.testclient import TestClient

    from barq_inference_b200.server.openai_api import OpenAIServer
    from barq_inference_b200.tokenizer.gguf_tokenizer import synthetic_tokenizer

    cfg = preset("tiny", n_layers=1, vocab=600, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=16)
    eng = _engine(cfg, t, num_blocks=64, max_num_batched_tokens=64)
    tok = synthetic_tokenizer(cfg.vocab)
    eng.tokenizer = tok
    srv = OpenAIServer(eng, tok)
    try:
        c = TestClient(srv.app)
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hello"}],
                                                  "max_tokens": 5, "temperature": 0})
        assert r.status_code == 200 and r.json()["choices"][0]["finish_reason"] in ("length", "stop")
        with c.stream("POST", "/v1/completions", json={"prompt": "the model", "max_tokens": 4, "stream": True}) as s:
            assert [ln for ln in s.iter_lines() if ln.startswith("data: ")][-1] == "data: [DONE]"
        h = c.get("/health").json()
        assert h["status"] == "ok" and 0 <= h["kv_usage"] <= 1
        m = c.get("/metrics").text
        assert "barq_kv_blocks_total 64" in m and "barq_requests_successful 2" in m
    finally:
        srv.aengine.shutdown()


def test_engine_step_failure_fails_in_flight_requests_and_recovers():
    """A step that raises (injected on the host, no device involved) fails the requests in flight;
    the engine thread keeps serving and the next request completes."""
    from barq_inference_b200.server.async_engine import AsyncEngine

    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=17)
    eng = _engine(cfg, t, num_blocks=64)
    real = eng.runner.forward
    calls = {"n": 0}

    def flaky(inp):
        calls["n"] += 1
        if calls["n"] == 2:
            raise RuntimeError("injected step failure")
        return real(inp)

    eng.runner.forward = flaky
    ae = AsyncEngine(eng)
    try:
        p = SamplingParams.greedy_params(max_tokens=5)
        items = list(ae.generate_blocking([1, 2, 3], p, timeout=60))
        assert items[-1].token is None and items[-1].finish_reason == "error"
        assert not ae.healthy and "injected" in ae.last_error
        assert eng.blocks.n_used == 1  # the failed sequence's pages went back to the pool
        items = list(ae.generate_blocking([4, 5, 6], p, timeout=60))
        assert [i.token is not None for i in items].count(True) == 5 and items[-1].finish_reason == "length"
        assert ae.healthy
    finally:
        ae.shutdown()


@pytest.mark.parametrize("window", [0, 24])
def test_decode_graph_path_host_side_matches_reference(window):
    """The CUDA-graph decode path without the graph: packed per-step inputs (incremental
    ``_Packed.fill``, rewritten rows after window trimming), padding rows, bucket sizes and the
    captured forward run eagerly on CPU."""
    import types

    from barq_inference_b200.engine.engine import _GraphBucket, _Packed

    class GraphOnCPU(Engine):
        def _run_decode(self, plan):
            B = next(b for b in self.ecfg.graph_buckets if b >= len(plan.seqs))
            return self._decode_graph(plan.seqs, B)

        def _capture(self, B):
            pk = _Packed(B, self.max_blocks_per_seq, self.device)
            gb = _GraphBucket()
            gb.B, gb.packed = B, pk
            gb.out_ids = torch.zeros(B, dtype=torch.int32)
            gb.graph = types.SimpleNamespace(replay=lambda: gb.out_ids.copy_(self._graph_forward(pk)))
            self.captured = getattr(self, "captured", 0) + 1
            return gb

    cfg = dataclasses.replace(preset("tiny", n_layers=1, vocab=400, max_ctx=256), sliding_window=window)
    t = random_tensors(cfg, POLICIES["tiny"], seed=18)
    ref = ReferenceModel(cfg, t)
    ec = EngineConfig(device="cpu", cuda_graphs=True, max_model_len=256, num_blocks=96, max_num_batched_tokens=48,
                      max_num_seqs=6, graph_buckets=(1, 2, 4, 8))
    eng = GraphOnCPU(cfg, t, ec, runner=PagedRefRunner(cfg, t))
    prompts = _prompts(cfg, 6, 19, lo=5, hi=40)
    params = [SamplingParams.greedy_params(max_tokens=n) for n in (3, 9, 17, 25, 6, 12)]  # rows leave at different steps
    res = eng.generate(prompts, params)
    assert eng.captured >= 3  # several buckets used as the batch shrinks
    assert (eng.sched.n_window_freed > 0) == bool(window)
    for p, r, sp in zip(prompts, res, params):
        assert len(r.tokens) == sp.max_tokens and _follows_reference(ref, p, r.tokens)


@pytest.mark.parametrize("kind", ["engine", "cpu"])
def test_model_context_encode_decode_truncate(kind):
    from barq_inference_b200.engine.context import ModelContext
    from barq_inference_b200.engine.cpu_engine import CPUEngine

    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=20)
    ref = ReferenceModel(cfg, t)
    eng = _engine(cfg, t, num_blocks=32) if kind == "engine" else CPUEngine(cfg, t, max_model_len=256)
    prompt = _prompts(cfg, 1, 21, lo=20, hi=21)[0]
    want = ref.forward(prompt)
    with ModelContext(eng) as ctx:
        allg = ctx.encode(prompt, all_logits=True)
        assert allg.shape == (len(prompt), cfg.vocab) and (allg - want).abs().max() < 1e-3
        tok = ctx.sample(allg[-1:], temperature=0.0)
        assert tok == int(want[-1].argmax())
        lg = ctx.decode(tok)
        assert (lg[0] - ref.forward(prompt + [tok])[-1]).abs().max() < 1e-3
        ctx.truncate(10)  # roll back and continue differently
        lg = ctx.encode([5, 6])
        assert (lg[0] - ref.forward(prompt[:10] + [5, 6])[-1]).abs().max() < 1e-3 and ctx.n_past == 12
    if kind == "engine":
        assert eng.blocks.n_used == 1  # pages returned


def test_stream_consumer_going_away_aborts_the_request():
    """An async stream closed early (a disconnected HTTP client) aborts its request on the engine
    thread: it stops generating and its pages return to the pool."""
    import asyncio
    import time

    from barq_inference_b200.server.async_engine import AsyncEngine

    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=22)
    eng = _engine(cfg, t, num_blocks=64)
    ae = AsyncEngine(eng)

    async def consume_two():
        agen = ae.stream([1, 2, 3], SamplingParams(max_tokens=200, temperature=0.0, ignore_eos=True))
        got = [await agen.__anext__(), await agen.__anext__()]
        await agen.aclose()
        return got

    try:
        got = asyncio.run(consume_two())
        assert all(g.token is not None for g in got)
        deadline = time.monotonic() + 30
        while (eng.sched.running or eng.sched.waiting) and time.monotonic() < deadline:
            time.sleep(0.01)
        assert not eng.sched.running and eng.blocks.n_used == 1
        assert eng.step_count < 150  # stopped long before its 200 tokens
    finally:
        ae.shutdown()


class PagedBuilder:
    """One rank's engine for multi-rank replica tests (picklable; patches the CPU sampler in the
    process it runs in)."""

    def __call__(self, device, rank, world):
        engine_mod.ops.sample = _greedy_sample
        cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
        return _engine(cfg, random_tensors(cfg, POLICIES["tiny"], seed=23), num_blocks=64)


def test_data_parallel_replicas_of_two_rank_groups():
    """--dp with --tp: each replica is a 2-rank lockstep group (rank 0 serves, rank 1 replays)."""
    from barq_inference_b200.parallel.dp import DataParallelEngine, TPReplicaFactory

    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    ref = ReferenceModel(cfg, random_tensors(cfg, POLICIES["tiny"], seed=23))
    front = DataParallelEngine(TPReplicaFactory(PagedBuilder(), 2), ["cpu", "cpu"], cfg=cfg, start_timeout=300)
    try:
        prompts = _prompts(cfg, 4, 24, lo=5, hi=20)
        outs = front.generate(prompts, SamplingParams.greedy_params(max_tokens=6))
        assert all(len(o) == 6 for o in outs)
        assert all(_follows_reference(ref, p, o) for p, o in zip(prompts, outs))
        assert all(r["served"] > 0 for r in front.replica_info())
    finally:
        front.shutdown()


def test_logprobs_of_the_rows_that_ask_for_them():
    """Rows with ``logprobs`` record log-softmax(raw logits)[token] (and the top alternatives) at every
    generated token, equal to the fp32 reference's; rows without it record nothing."""
    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=8)
    ref = ReferenceModel(cfg, t)
    eng = _engine(cfg, t, num_blocks=64, max_num_batched_tokens=128, max_num_seqs=4)
    prompts = _prompts(cfg, 3, 9)
    with_lp = dataclasses.replace(SamplingParams.greedy_params(max_tokens=6), logprobs=True, top_logprobs=3)
    params = [with_lp, SamplingParams.greedy_params(max_tokens=6), with_lp]
    res = eng.generate(prompts, params)
    assert res[1].logprobs == [] and res[1].top_logprobs == []
    for i in (0, 2):
        r = res[i]
        assert len(r.logprobs) == len(r.tokens) == 6 and all(len(x) == 3 for x in r.top_logprobs)
        cache: dict = {}
        logits = ref.forward(prompts[i], cache)[-1]
        for tok, lp, top in zip(r.tokens, r.logprobs, r.top_logprobs):
            lsm = torch.log_softmax(logits.float(), -1)
            assert abs(lp - float(lsm[tok])) < 1e-3
            assert [a for a, _ in top] == lsm.topk(3).indices.tolist()
            logits = ref.forward([tok], cache)[-1]


def test_prompt_lookup_speculation_follows_target_reference():
    """Drafts copied from earlier n-grams (no draft model): greedy output is the target's greedy
    continuation; on a repetitive context the drafts are accepted and fewer target steps run."""
    from barq_inference_b200.engine.speculative import SpeculativeConfig, SpeculativeDecoder, lookup_drafts

    assert lookup_drafts([1, 2, 3, 9, 1, 2, 3], 3) == [9, 1, 2]
    assert lookup_drafts([5, 6, 7], 2) == [] and lookup_drafts([4, 4], 2) == [4]
    assert lookup_drafts([1, 2, 8, 2, 9, 1, 2], 2, n_max=2) == [8, 2]  # longest match first
    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=13)
    ref = ReferenceModel(cfg, t)
    target = _engine(cfg, t, num_blocks=64)
    prompt = _prompts(cfg, 1, 15, lo=20, hi=21)[0]
    # make the context repeat the model's own greedy continuation: the lookup then finds it
    cache: dict = {}
    logits = ref.forward(prompt, cache)[-1]
    cont = []
    for _ in range(12):
        cont.append(int(logits.argmax()))
        logits = ref.forward([cont[-1]], cache)[-1]
    ctx = prompt + cont + prompt
    p = SamplingParams.greedy_params(max_tokens=12)
    res = SpeculativeDecoder(target, None, SpeculativeConfig(6)).generate(ctx, p)
    assert len(res.tokens) == 12 and _follows_reference(ref, ctx, res.tokens)
    assert res.stats.accepted > 0 and res.stats.steps < 12
    assert target.blocks.n_used == 1
    # sampled decoding stays within the target's support (drafts are one-hot proposals)
    ps = dataclasses.replace(SamplingParams(temperature=0.8, top_k=5, seed=3), max_tokens=10)
    res = SpeculativeDecoder(target, None, SpeculativeConfig(4)).generate(ctx, ps)
    assert len(res.tokens) == 10
