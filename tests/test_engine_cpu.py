"""Host-side engine logic: block manager, scheduler, reference model (CPU)."""
import torch

from barq_inference_b200.engine.kv_cache import BlockManager, OutOfBlocks
from barq_inference_b200.engine.sampling_params import SamplingParams
from barq_inference_b200.engine.scheduler import Scheduler, SchedulerConfig
from barq_inference_b200.engine.sequence import Sequence
from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.models.reference import ReferenceModel


def test_block_manager():
    bm = BlockManager(10)
    a = bm.allocate(3)
    bm.retain(a[:1])
    bm.release(a)
    assert bm.n_free == 9
    bm.release(a[:1])
    assert bm.n_free == 10
    try:
        bm.allocate(11)
        assert False
    except OutOfBlocks:
        pass
    t = []
    bm.grow(t, 33)
    assert len(t) == 3


def test_scheduler_prefill_then_decode_and_chunking():
    bm = BlockManager(100)
    s = Scheduler(SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=40, max_model_len=512), bm)
    seqs = [Sequence(list(range(30)), SamplingParams()) for _ in range(3)]
    for q in seqs:
        s.add(q)
    st = s.schedule()
    assert st.kind == "prefill" and st.n_new == [30, 10]
    for q, n in zip(st.seqs, st.n_new):
        q.n_cached += n
    st = s.schedule()  # continue the chunked prompt, admit the third
    assert st.kind == "prefill" and st.seqs[0] is seqs[1] and st.n_new[0] == 20
    for q, n in zip(st.seqs, st.n_new):
        q.n_cached += n
    st = s.schedule()
    assert st.kind == "prefill" and st.seqs == [seqs[2]] or st.kind == "prefill"


def test_scheduler_preempts_youngest():
    bm = BlockManager(6)
    s = Scheduler(SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=1000, max_model_len=512), bm)
    a, b = Sequence(list(range(32)), SamplingParams()), Sequence(list(range(32)), SamplingParams())
    s.add(a)
    s.add(b)
    st = s.schedule()
    assert st.kind == "prefill" and len(st.seqs) == 2
    for q in st.seqs:
        q.n_cached = 32
        q.output.append(1)
    bm.allocate(bm.n_free)  # exhaust the pool
    st = s.schedule()
    assert st.kind == "decode" and st.seqs == [a]
    assert b in s.waiting and b.n_preempted == 1 and not b.block_table


def test_reference_tiny_deterministic():
    cfg = preset("tiny")
    t = random_tensors(cfg, POLICIES["tiny"], seed=0)
    m = ReferenceModel(cfg, t)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab, (64,), generator=g).tolist()
    a, _ = m.greedy(prompt, 6)
    b, _ = ReferenceModel(cfg, t).greedy(prompt, 6)
    assert a == b
    # incremental decode == full recompute
    full = m.forward(prompt + a[:3])[-1]
    cache = {}
    m.forward(prompt, cache)
    for tok in a[:2]:
        m.forward([tok], cache)
    inc = m.forward([a[2]], cache)[-1]
    assert torch.allclose(full, inc, atol=1e-4)


def test_scheduler_sliding_window_frees_dead_blocks():
    """With a 32-token window, blocks wholly behind every future query's window go back to the pool
    (their table entries name the dummy block); a long generation keeps a bounded block count."""
    bm = BlockManager(64)
    dummy = bm.allocate(1)[0]
    s = Scheduler(SchedulerConfig(max_num_seqs=2, max_num_batched_tokens=48, max_model_len=4096, sliding_window=32), bm)
    s.dummy_block = dummy
    q = Sequence(list(range(100)), SamplingParams())
    s.add(q)
    peak = 0
    for step in range(300):
        st = s.schedule()
        assert st is not None
        for x, n in zip(st.seqs, st.n_new):
            x.n_cached += n
            if x.n_cached >= x.n_tokens:
                x.output.append(7)
        peak = max(peak, bm.n_used)
        live = [b for b in q.block_table[q.window_freed:]]
        assert dummy not in live and all(b == dummy for b in q.block_table[:q.window_freed])
        # every position a future query can attend to is still backed by a live block
        first_needed = max(0, q.n_cached - 32 + 1)
        assert q.window_freed <= first_needed // 16
    assert q.n_tokens > 350 and s.n_window_freed >= 18
    assert peak <= 1 + (48 + 32) // 16 + 2, peak  # dummy + window + one prefill chunk, not the sequence
    s.finish(q, "length")
    assert bm.n_used == 1  # only the dummy block: no double free, nothing leaked


def test_scheduler_admission_control():
    """Refused up front: a prompt larger than the whole KV pool (it could never be scheduled), and
    requests beyond the waiting-queue limit (Overloaded, which servers turn into 503)."""
    import pytest

    from barq_inference_b200.engine.scheduler import Overloaded

    bm = BlockManager(8)
    s = Scheduler(SchedulerConfig(max_num_seqs=2, max_num_batched_tokens=64, max_model_len=4096, max_waiting=2), bm)
    s.dummy_block = bm.allocate(1)[0]
    with pytest.raises(ValueError, match="KV pages"):
        s.add(Sequence(list(range(7 * 16)), SamplingParams()))  # needs 8 pages, 7 usable
    s.add(Sequence([1, 2, 3], SamplingParams()))
    s.add(Sequence([1, 2, 3], SamplingParams()))
    with pytest.raises(Overloaded):
        s.add(Sequence([1, 2, 3], SamplingParams()))
    s.schedule()  # admits the waiting ones; the queue has room again
    s.add(Sequence([4, 5], SamplingParams()))


def test_http_503_when_overloaded():
    from fastapi.testclient import TestClient

    from barq_inference_b200.engine.cpu_engine import CPUEngine
    from barq_inference_b200.server.openai_api import OpenAIServer
    from barq_inference_b200.tokenizer.gguf_tokenizer import synthetic_tokenizer

    cfg = preset("tiny", n_layers=1, vocab=600, max_ctx=256)
    eng = CPUEngine(cfg, random_tensors(cfg, POLICIES["tiny"], seed=0), max_model_len=256, max_waiting=1)
    eng.waiting.append(Sequence([1, 2], SamplingParams()))  # a request already queued ...
    eng.has_work = lambda: False  # ... that the engine thread leaves there
    srv = OpenAIServer(eng, synthetic_tokenizer(cfg.vocab))
    try:
        r = TestClient(srv.app).post("/v1/completions", json={"prompt": "hi", "max_tokens": 2})
        assert r.status_code == 503 and r.json()["error"]["type"] == "overloaded_error"
    finally:
        srv.aengine.shutdown()


def test_incremental_decode_packing_equals_full_rewrite():
    """The decode graph's packed host inputs, written incrementally (only appended block-table
    entries for a row whose sequence is unchanged), are byte-identical to rewriting every array each
    step — across joins, departures, preemption (table replaced), window trimming and growth."""
    import random
    import types

    import numpy as np

    from barq_inference_b200.engine.engine import Engine, _Packed

    rng = random.Random(0)
    B, mb, bs, dummy = 8, 32, 16, 0
    eng = Engine.__new__(Engine)
    eng.ecfg = types.SimpleNamespace(block_size=bs)
    eng.dummy_block, eng.max_blocks_per_seq = dummy, mb
    inc, ref = _Packed(B, mb, "cpu"), _Packed(B, mb, "cpu")
    pool = []
    nxt = iter(range(1, 10**6))

    def new_seq():
        s = Sequence([rng.randrange(100) for _ in range(rng.randint(1, 40))],
                     SamplingParams(temperature=rng.choice([0.0, 0.7]), top_k=rng.choice([0, 40]), seed=rng.randint(0, 3)))
        s.block_table = [next(nxt) for _ in range((s.n_tokens + bs - 1) // bs)]
        return s

    for step in range(400):
        if len(pool) < B and rng.random() < 0.3:
            pool.insert(rng.randrange(len(pool) + 1), new_seq())
        if pool and rng.random() < 0.1:
            pool.pop(rng.randrange(len(pool)))
        for s in pool:
            s.output.append(rng.randrange(100))
            while len(s.block_table) * bs < s.n_tokens:
                s.block_table.append(next(nxt))
        if pool and rng.random() < 0.05:  # preempted and readmitted: a new table of the same length
            s = rng.choice(pool)
            s.block_table = [next(nxt) for _ in s.block_table]
            s.bt_gen += 1
        if pool and rng.random() < 0.05:  # sliding window: leading entries point at the dummy page
            s = rng.choice(pool)
            k = rng.randint(0, len(s.block_table) - 1)
            s.block_table[:k] = [dummy] * k
            s.bt_gen += 1
        if not pool:
            continue
        n = inc.fill(pool, bs, dummy)
        ids, pos, slots, lens, bt, _ = eng._decode_arrays(pool, B)
        temp, topk, topp, minp, seeds, steps = eng._sampling_tensors(pool, B)
        for k, a in (("ids", ids), ("pos", pos), ("slots", slots), ("lens", lens), ("bt", bt), ("temp", temp),
                     ("topk", topk), ("topp", topp), ("minp", minp), ("seeds", seeds), ("steps", steps)):
            ref.h[k][...] = a
        assert n == len(pool)
        assert np.array_equal(inc.host.numpy(), ref.host.numpy()), step


def test_prefill_arrays_match_per_token_construction():
    import random
    import types

    import numpy as np

    from barq_inference_b200.engine.engine import Engine
    from barq_inference_b200.engine.scheduler import ScheduledStep

    rng = random.Random(1)
    eng = Engine.__new__(Engine)
    eng.ecfg = types.SimpleNamespace(block_size=16)
    for trial in range(50):
        seqs, n_new = [], []
        for _ in range(rng.randint(1, 5)):
            s = Sequence([rng.randrange(1000) for _ in range(rng.randint(1, 90))], SamplingParams())
            s.output = [rng.randrange(1000) for _ in range(rng.choice([0, 0, 3]))]
            s.n_cached = rng.randint(0, s.n_tokens - 1)
            n = rng.randint(1, s.n_tokens - s.n_cached)
            s.block_table = rng.sample(range(1, 500), (s.n_cached + n + 15) // 16)
            if rng.random() < 0.3:
                st = rng.randrange(len(s.prompt))
                s.embeds = (st, torch.randn(min(5, len(s.prompt) - st), 8))
            seqs.append(s)
            n_new.append(n)
        ids, pos, slots, qs, last, bt, lens, e_rows, e_vals = eng._prefill_arrays(ScheduledStep("prefill", seqs, n_new))
        want_ids, want_pos, want_slots, want_rows = [], [], [], []
        for s, n in zip(seqs, n_new):
            if s.embeds is not None:
                st, e = s.embeds
                for p in range(max(st, s.n_cached), min(st + e.shape[0], s.n_cached + n)):
                    want_rows.append(len(want_ids) + p - s.n_cached)
            for p in range(s.n_cached, s.n_cached + n):
                want_ids.append(s.tokens[p])
                want_pos.append(p)
                want_slots.append(s.block_table[p // 16] * 16 + p % 16)
        assert ids.dtype == np.int32 and pos.dtype == np.int32 and slots.dtype == np.int64
        assert ids.tolist() == want_ids and pos.tolist() == want_pos and slots.tolist() == want_slots
        assert qs.tolist() == [0] + list(np.cumsum(n_new)) and last.tolist() == [q - 1 for q in qs.tolist()[1:]]
        assert e_rows == want_rows and lens.tolist() == [s.n_cached + n for s, n in zip(seqs, n_new)]


def test_embed_gpu_plumbing_with_stub_runner():
    """The GPU engine's embedding path (chunked prefill on borrowed pages, hidden-row tap, output norm,
    mean pooling) driven by a stub runner on CPU tensors: pages go back to the pool, chunking does not
    change the result, StepInputs carry consistent positions and slots."""
    import types

    from barq_inference_b200.engine.embeddings import embed_gpu
    from barq_inference_b200.models.runner import LlamaRunner

    H = 8
    seen = []

    def fwd(inp):
        seen.append((inp.pos.tolist(), inp.slots.tolist(), inp.block_tables.tolist()))
        ids = inp.ids.to(torch.float32)
        inp.hidden_out.copy_(torch.stack([ids * (k + 1) + 1.0 for k in range(H)], 1))

    r = LlamaRunner.__new__(LlamaRunner)
    r.pp, r.comm, r.out_norm = None, None, torch.full((H,), 2.0)
    r.forward = fwd
    bm = BlockManager(16, 4)
    res = []
    for step in (3, 100):
        eng = types.SimpleNamespace(runner=r, cfg=types.SimpleNamespace(hidden=H, rms_eps=1e-6), blocks=bm,
                                    prefix_cache=None, device=torch.device("cpu"),
                                    ecfg=types.SimpleNamespace(block_size=4, max_model_len=64, max_num_batched_tokens=step))
        res.append(embed_gpu(eng, [[1, 2, 3, 4, 5, 6, 7], [9]]))
        assert bm.n_used == 0
    assert torch.allclose(res[0], res[1], atol=1e-6)
    x = torch.stack([torch.tensor([1., 2, 3, 4, 5, 6, 7]) * (k + 1) + 1 for k in range(H)], 1)
    h = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * 2.0
    want = h.mean(0) / h.mean(0).norm()
    assert torch.allclose(res[1][0], want, atol=1e-6)
    pos, slots, bt = seen[1]  # second chunk of the first prompt with step 3: positions 3..5
    assert pos == [3, 4, 5] and slots == [bt[0][p // 4] * 4 + p % 4 for p in pos]
