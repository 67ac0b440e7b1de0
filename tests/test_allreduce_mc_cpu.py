"""CPU model of the NVLS (multimem) form of the one-shot all-reduce (``allreduce_add_mc_kernel`` in
``csrc/kernels/allreduce.cu``): the kernel's slice and grid-stride index arithmetic, run for every
(rank, block, thread), must reduce every float4 exactly once, write the sum back to every rank,
and let each block's final pass read only positions that its own barrier covers (the same block of
every rank wrote them).  Every rank must end with the same x + sum of partials."""
import itertools

import numpy as np
import pytest

THREADS = 256


def slices(n4, world, rank):
    S = (n4 + world - 1) // world
    lo = min(n4, rank * S)
    return lo, min(n4, lo + S), S


def run_model(n, world, blocks, rng):
    n4 = n // 4
    parts = [rng.standard_normal(n).astype(np.float32) for _ in range(world)]
    xs = [rng.standard_normal(n).astype(np.float32) for _ in range(world)]
    bufs = [p.copy() for p in parts]
    stride = blocks * THREADS
    writer = {}  # float4 index -> (rank, block) that reduced it
    # step 2: rank r, block b reduces its slice positions and writes the sum to every rank
    for r, b in itertools.product(range(world), range(blocks)):
        lo, hi, _ = slices(n4, world, r)
        for t in range(THREADS):
            for i in range(lo + b * THREADS + t, hi, stride):
                assert i not in writer, "a float4 reduced twice"
                writer[i] = (r, b)
                s = np.sum(np.stack([parts[q][4 * i:4 * i + 4] for q in range(world)]), axis=0, dtype=np.float32)
                for q in range(world):
                    bufs[q][4 * i:4 * i + 4] = s
    assert set(writer) == set(range(n4)), "float4 positions missing"
    # step 4: each rank's block b reads the positions of every rank's slice at its own (block, thread)
    outs = []
    for q in range(world):
        x = xs[q].copy()
        seen = set()
        for b in range(blocks):
            for r in range(world):
                lo, hi, _ = slices(n4, world, r)
                for t in range(THREADS):
                    for i in range(lo + b * THREADS + t, hi, stride):
                        assert writer[i][1] == b, "read a position another block's barrier does not cover"
                        seen.add(i)
                        x[4 * i:4 * i + 4] += bufs[q][4 * i:4 * i + 4]
        assert seen == set(range(n4))
        for i in range(n4 * 4, n):  # tail: rank-order sum from peer memory (block 0)
            acc = x[i]
            for r in range(world):
                acc = np.float32(acc + parts[r][i])
            x[i] = acc
        outs.append(x)
    return xs, parts, outs, bufs


@pytest.mark.parametrize("n,world,blocks", [(4096, 2, 4), (4096 * 3 + 8, 8, 32), (1000, 4, 3), (37, 8, 1),
                                             (14336, 8, 32)])
def test_multimem_allreduce_index_model(n, world, blocks):
    rng = np.random.default_rng(n + world)
    xs, parts, outs, bufs = run_model(n, world, blocks, rng)
    ref = [x.astype(np.float64) + np.sum(np.stack(parts).astype(np.float64), axis=0) for x in xs]
    for q in range(world):
        np.testing.assert_allclose(outs[q], ref[q], rtol=1e-5, atol=1e-5)
    # every rank holds the same (bit-identical) reduced sums after the write-back
    n4 = n // 4
    for q in range(1, world):
        np.testing.assert_array_equal(bufs[q][:4 * n4], bufs[0][:4 * n4])
