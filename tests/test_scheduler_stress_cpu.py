"""Randomized scheduler runs (continuous batching, chunked prefill, preemption under a small KV pool,
radix prefix cache with shared prompt prefixes, sliding-window page freeing): every request finishes
with exactly its token budget, page reference counts always equal the references held, no page is
freed twice or leaked."""
import random
from collections import Counter

import pytest

from barq_inference_b200.engine.kv_cache import BlockManager
from barq_inference_b200.engine.prefix_cache import RadixPrefixCache
from barq_inference_b200.engine.sampling_params import SamplingParams
from barq_inference_b200.engine.scheduler import Scheduler, SchedulerConfig
from barq_inference_b200.engine.sequence import SeqStatus, Sequence


def _check_refs(bm: BlockManager, sched: Scheduler, cache, dummy):
    held = Counter()
    for s in sched.running:
        for i, b in enumerate(s.block_table):
            if i >= s.window_freed:
                held[b] += 1
    if cache is not None:
        stack = [cache.root]
        while stack:
            nd = stack.pop()
            if nd is not cache.root:
                held[nd.block] += 1
            stack.extend(nd.children.values())
    held[dummy] += 1
    for b in range(bm.num_blocks):
        assert bm.ref[b] == held[b], (b, bm.ref[b], held[b])
    assert len(set(bm.free)) == len(bm.free) and all(bm.ref[b] == 0 for b in bm.free)


@pytest.mark.parametrize("seed,prefix,window", [(0, False, 0), (1, True, 0), (2, False, 40), (3, True, 0),
                                                (4, True, 24), (5, False, 0)])
def test_random_workload_invariants(seed, prefix, window):
    rng = random.Random(seed)
    bm = BlockManager(rng.choice([24, 40, 64]))
    cache = RadixPrefixCache(bm) if prefix else None
    sched = Scheduler(SchedulerConfig(max_num_seqs=rng.choice([2, 4, 8]), max_num_batched_tokens=rng.choice([16, 48, 96]),
                                      max_model_len=512, sliding_window=window), bm, cache)
    dummy = bm.allocate(1)[0]
    sched.dummy_block = dummy
    shared = [rng.randrange(1000) for _ in range(40)]
    pending = []
    for _ in range(30):
        base = shared[: rng.choice([0, 16, 32, 40])] if prefix else []
        prompt = base + [rng.randrange(1000) for _ in range(rng.randint(1, 60))]
        pending.append(Sequence(prompt, SamplingParams(max_tokens=rng.randint(1, 40))))
    finished = []
    steps = 0
    while pending or sched.has_work:
        if pending and rng.random() < 0.4:
            sched.add(pending.pop(0))
        st = sched.schedule()
        steps += 1
        assert steps < 20000
        if st is None:
            assert not sched.running or sched.waiting
            if not pending and not sched.running and sched.waiting:
                raise AssertionError("waiting requests that can never be admitted")
            continue
        assert len(st.seqs) == len(set(id(s) for s in st.seqs))
        for s, n in zip(st.seqs, st.n_new):
            assert s.status is SeqStatus.RUNNING
            assert len(s.block_table) * bm.block_size >= s.n_cached + n  # pages cover what is written
            s.n_cached += n
            if s.n_cached >= s.n_tokens:
                s.output.append(rng.randrange(1000))
                if len(s.output) >= s.params.max_tokens:
                    sched.finish(s, "length")
                    finished.append(s)
        _check_refs(bm, sched, cache, dummy)
    assert len(finished) == 30 and all(len(s.output) == s.params.max_tokens for s in finished)
    assert all(not s.block_table for s in finished)
    if cache is not None:
        assert bm.n_used == 1 + cache.n_blocks  # the dummy page plus what the prefix cache keeps
        cache.evict(bm.num_blocks)
    assert bm.n_used == 1
