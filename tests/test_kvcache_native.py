"""The C++ KV block pool and radix prefix cache (csrc/native/kvcache_native.cpp) against the Python
implementations (engine/kv_cache.py, engine/prefix_cache.py) on random operation sequences: same
block ids, reference counts, free lists, prefix matches and LRU evictions."""
import random

import pytest

from barq_inference_b200.engine.kv_cache import BlockManager, NativeBlockManager, OutOfBlocks, _native_kv
from barq_inference_b200.engine.prefix_cache import NativeRadixPrefixCache, RadixPrefixCache

pytestmark = pytest.mark.skipif(_native_kv() is None, reason="barq_inference_b200._native not built")


def _same(py, nat):
    assert py.n_free == nat.n_free and py.n_used == nat.n_used
    assert list(py.ref) == list(nat.ref)
    assert list(py.free) == list(nat.free)


@pytest.mark.parametrize("seed", range(6))
def test_random_sequences_match_the_python_oracle(seed):
    rng = random.Random(seed)
    nb, bs = rng.choice([(24, 4), (64, 16), (40, 8)])
    py, nat = BlockManager(nb, bs), NativeBlockManager(nb, bs)
    pc, nc = RadixPrefixCache(py), NativeRadixPrefixCache(nat)
    vocab = 3  # a tiny vocabulary makes shared prefixes (and tree hits) common
    held: list[list[int]] = []  # block tables of "running sequences"
    for _ in range(400):
        op = rng.random()
        if op < 0.3:  # a new sequence: match a prompt, retain the hit, grow the rest
            toks = [rng.randrange(vocab) for _ in range(rng.randrange(1, 6 * bs))]
            a, b = pc.match(toks), nc.match(toks)
            assert a == b
            blocks, n = a
            need = py.blocks_for(len(toks) + 1) - len(blocks)
            if not py.can_allocate(need):
                assert nat.can_allocate(need) is False
                assert pc.evict(need - py.n_free) == nc.evict(need - nat.n_free)
                _same(py, nat)
                continue
            py.retain(blocks)
            nat.retain(blocks)
            t1, t2 = list(blocks), list(blocks)
            assert py.grow(t1, len(toks) + 1) == nat.grow(t2, len(toks) + 1)
            held.append((toks, t1))
        elif op < 0.55 and held:  # a sequence finishes: donate its full blocks, release its table
            toks, table = held.pop(rng.randrange(len(held)))
            pc.insert(toks, table)
            nc.insert(toks, table)
            py.release(table)
            nat.release(table)
        elif op < 0.7:
            n = rng.randrange(1, 8)
            assert pc.evict(n) == nc.evict(n)
        elif op < 0.85:
            n = rng.randrange(1, 6)
            if py.can_allocate(n):
                a, b = py.allocate(n), nat.allocate(n)
                assert a == b
                py.release(a)
                nat.release(b)
            else:
                with pytest.raises(OutOfBlocks):
                    nat.allocate(n)
        else:
            toks = [rng.randrange(vocab) for _ in range(rng.randrange(1, 4 * bs))]
            assert pc.match(toks) == nc.match(toks)
        _same(py, nat)
        assert pc.n_blocks == nc.n_blocks and pc.hits == nc.hits and pc.queries == nc.queries


def test_errors_match():
    nat = NativeBlockManager(4, 16)
    with pytest.raises(ValueError):
        nat.release([1])
    with pytest.raises(ValueError):
        nat.retain([2])
    with pytest.raises(OutOfBlocks):
        nat.allocate(5)
    with pytest.raises(IndexError):
        nat.retain([9])
