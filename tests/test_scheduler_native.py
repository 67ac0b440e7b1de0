"""The native scheduler core (``csrc/native/scheduler_native.cpp`` through ``NativeScheduler``)
against the Python ``Scheduler`` on the same random workloads: continuous batching, chunked
prefill, preemption under a small pool, prefix-cache hits and evictions, sliding-window page
release, embedding prompts, aborts and queue clearing.  Every step must give the same plan (kind,
sequences, token counts), the same block tables and the same pool state."""
import random

import pytest

torch = pytest.importorskip("torch")

from barq_inference_b200.engine.kv_cache import BlockManager, NativeBlockManager, _native_kv  # noqa: E402
from barq_inference_b200.engine.prefix_cache import NativeRadixPrefixCache, RadixPrefixCache  # noqa: E402
from barq_inference_b200.engine.sampling_params import SamplingParams  # noqa: E402
from barq_inference_b200.engine.scheduler import (NativeScheduler, Overloaded, Scheduler,  # noqa: E402
                                                  SchedulerConfig, new_scheduler)
from barq_inference_b200.engine.sequence import SeqStatus, Sequence  # noqa: E402

pytestmark = pytest.mark.skipif(_native_kv() is None, reason="native extension not built")


def _pair(num_blocks, cfg, prefix):
    py_bm, nat_bm = BlockManager(num_blocks), NativeBlockManager(num_blocks)
    py_pc = RadixPrefixCache(py_bm) if prefix else None
    nat_pc = NativeRadixPrefixCache(nat_bm) if prefix else None
    py, nat = Scheduler(cfg, py_bm, py_pc), NativeScheduler(cfg, nat_bm, nat_pc)
    for bm, s in ((py_bm, py), (nat_bm, nat)):
        s.dummy_block = bm.allocate(1)[0]
    return (py, py_bm, py_pc), (nat, nat_bm, nat_pc)


def _same_state(py, py_bm, nat, nat_bm, twins):
    assert py_bm.free == nat_bm.free and py_bm.ref == nat_bm.ref
    assert [twins[id(s)] for s in py.waiting] == [s.seq_id for s in nat.waiting]
    assert [twins[id(s)] for s in py.running] == [s.seq_id for s in nat.running]
    assert (py.n_preemptions, py.n_window_freed) == (nat.n_preemptions, nat.n_window_freed)


@pytest.mark.parametrize("seed,prefix,window,tight", [(0, False, 0, False), (1, True, 0, False), (2, False, 40, False),
                                                      (3, True, 0, False), (4, True, 24, False), (5, False, 0, False),
                                                      (6, True, 0, False), (7, True, 32, False), (8, False, 16, False),
                                                      (9, True, 0, False), (10, False, 0, True), (11, True, 0, True),
                                                      (12, False, 24, True), (13, True, 0, True), (14, False, 0, True)])
def test_native_scheduler_matches_python(seed, prefix, window, tight):
    """``tight``: a pool of 12-16 pages under 8 long generations, so that decode steps and prefill
    chunks preempt (and the prefix cache evicts)."""
    rng = random.Random(seed)
    cfg = SchedulerConfig(max_num_seqs=8 if tight else rng.choice([2, 4, 8]),
                          max_num_batched_tokens=rng.choice([16, 48, 96]),
                          max_model_len=512, sliding_window=window, chunked_prefill=tight or rng.random() < 0.8)
    (py, py_bm, py_pc), (nat, nat_bm, nat_pc) = _pair(rng.choice([12, 16] if tight else [24, 40, 64]), cfg, prefix)
    shared = [rng.randrange(1000) for _ in range(40)]
    pending = []
    for i in range(40):
        base = shared[: rng.choice([0, 16, 32, 40])] if prefix else []
        prompt = base + [rng.randrange(1000) for _ in range(rng.randint(1, 60))]
        params = SamplingParams(max_tokens=rng.randint(40, 100) if tight else rng.randint(1, 40))
        arrival = float(i // 3)  # ties exercise the first-in-running-order rule of preemption
        embeds = "rows" if rng.random() < 0.1 else None
        pending.append((Sequence(list(prompt), params, arrival=arrival, embeds=embeds),
                        Sequence(list(prompt), params, arrival=arrival, embeds=embeds)))
    twins = {id(a): b.seq_id for a, b in pending}
    by_nat = {b.seq_id: a for a, b in pending}
    live = []
    steps = 0
    while pending or py.has_work:
        assert nat.has_work == py.has_work or pending
        r = rng.random()
        if pending and r < 0.4:
            a, b = pending.pop(0)
            py.add(a)
            nat.add(b)
            live.append((a, b))
        elif live and r < 0.45:  # a client goes away
            a, b = live.pop(rng.randrange(len(live)))
            assert py.abort(a) == nat.abort(b)
        ps, ns = py.schedule(), nat.schedule()
        steps += 1
        assert steps < 20000
        _same_state(py, py_bm, nat, nat_bm, twins)
        if ps is None:
            assert ns is None
            if not pending and py.waiting and not py.running:
                py.clear_waiting()
                nat.clear_waiting()
            continue
        assert ns is not None and ps.kind == ns.kind and ps.n_new == ns.n_new
        assert [twins[id(s)] for s in ps.seqs] == [s.seq_id for s in ns.seqs]
        for a, b, n in zip(ps.seqs, ns.seqs, ps.n_new):
            assert b.status is SeqStatus.RUNNING and a.status is SeqStatus.RUNNING
            assert a.block_table == b.block_table and a.n_cached == b.n_cached
            assert (a.window_freed, a.prefix_hit, a.n_preempted) == (b.window_freed, b.prefix_hit, b.n_preempted)
            for s in (a, b):
                s.n_cached += n
            if a.n_cached >= a.n_tokens:
                tok = rng.randrange(1000)
                a.output.append(tok)
                b.output.append(tok)
                if len(a.output) >= a.params.max_tokens:
                    py.finish(a, "length")
                    nat.finish(b, "length")
                    assert not b.block_table and b.status is SeqStatus.FINISHED and b.finish_reason == "length"
        _same_state(py, py_bm, nat, nat_bm, twins)
    assert all(a.status is SeqStatus.FINISHED for a in by_nat.values())
    if tight and not window:
        assert nat.n_preemptions > 0
    if prefix:
        assert py_pc.n_blocks == nat_pc.n_blocks
        assert py_pc.evict(10**6) == nat_pc.evict(10**6)
    assert py_bm.n_used == nat_bm.n_used == 1


def test_native_scheduler_admission_errors_and_factory(monkeypatch):
    bm = NativeBlockManager(8)
    s = new_scheduler(SchedulerConfig(max_num_seqs=2, max_num_batched_tokens=64, max_model_len=200, max_waiting=1),
                      bm)
    assert isinstance(s, NativeScheduler)
    s.dummy_block = bm.allocate(1)[0]
    with pytest.raises(ValueError, match="empty prompt"):
        s.add(Sequence([], SamplingParams()))
    with pytest.raises(ValueError, match="max_model_len"):
        s.add(Sequence(list(range(200)), SamplingParams()))
    with pytest.raises(ValueError, match="KV pages"):
        s.add(Sequence(list(range(150)), SamplingParams()))  # 10 pages; 7 usable besides the dummy
    a = Sequence([1, 2, 3], SamplingParams())
    s.add(a)
    with pytest.raises(Overloaded):
        s.add(Sequence([4], SamplingParams()))
    st = s.schedule()
    assert st.kind == "prefill" and st.seqs == [a] and a.block_table and a.status is SeqStatus.RUNNING
    assert s.abort(a) and not s.abort(a) and a.finish_reason == "abort" and bm.n_used == 1
    assert not s.has_work
    # the Python class whenever any piece is Python, or on request
    assert isinstance(new_scheduler(SchedulerConfig(), BlockManager(8)), Scheduler)
    assert isinstance(new_scheduler(SchedulerConfig(), bm, RadixPrefixCache(BlockManager(8))), Scheduler)
    monkeypatch.setenv("BARQ_NATIVE_SCHED", "0")
    assert isinstance(new_scheduler(SchedulerConfig(), bm), Scheduler)


@pytest.mark.parametrize("native", [False, True])
def test_prefill_phase_never_preempts_a_sequence_already_in_the_plan(native):
    """Two running sequences each carrying several unprocessed tokens (speculative decoding appends
    more than one per step) are both continued in the prefill phase.  When the second needs a page
    and the pool is dry, the only younger sequence is the first, which is already in this step's
    plan: it must not be preempted (its pages would be freed under the step); the second waits."""
    bm = NativeBlockManager(3) if native else BlockManager(3)  # the dummy page + 2 usable
    cls = NativeScheduler if native else Scheduler
    s = cls(SchedulerConfig(max_num_seqs=4, max_num_batched_tokens=64, max_model_len=64), bm)
    s.dummy_block = bm.allocate(1)[0]
    young = Sequence(list(range(10)), SamplingParams(), arrival=5.0)
    old = Sequence(list(range(16)), SamplingParams(), arrival=1.0)
    s.add(young)
    s.add(old)
    st = s.schedule()
    assert st.kind == "prefill" and st.seqs == [young, old] and st.n_new == [10, 16]
    for q, n in zip(st.seqs, st.n_new):
        q.n_cached += n
        q.output.extend([7, 8, 9])  # three accepted tokens: young stays inside its page, old does not
    st = s.schedule()
    assert st.kind == "prefill" and st.seqs == [young] and st.n_new == [3]
    assert young.status is SeqStatus.RUNNING and len(young.block_table) == 1
    assert old.status is SeqStatus.RUNNING and s.n_preemptions == 0


@pytest.mark.parametrize("native", [False, True])
def test_finishing_a_waiting_sequence_removes_it_from_the_queue(native):
    bm = NativeBlockManager(8) if native else BlockManager(8)
    s = (NativeScheduler if native else Scheduler)(SchedulerConfig(max_num_seqs=1, max_num_batched_tokens=64), bm)
    a, b = Sequence([1, 2, 3], SamplingParams()), Sequence([4, 5], SamplingParams())
    s.add(a)
    s.add(b)
    assert s.schedule().seqs == [a]  # b waits: one sequence at a time
    s.finish(b, "error")
    assert b.status is SeqStatus.FINISHED and b not in s.waiting and len(s.waiting) == 0
    s.finish(a, "length")
    assert not s.has_work and bm.n_used == 0
