"""The fused push all-reduce protocol on a CPU loopback fabric (one thread per rank): random per-rank
delays, bit-identical sums across ranks, bounded waits that keep epochs aligned, and the buffer reuse
rule (reuse without an intervening collective ends in a timeout, never in a wrong sum)."""
import numpy as np
import pytest

from barq_inference_b200.parallel.loopback import LoopbackFabric, run_ranks


def _parts(world, B, N, seed):
    g = np.random.default_rng(seed)
    return [(g.standard_normal((B, N)) * 10 ** g.uniform(-3, 3, (B, N))).astype(np.float32) for _ in range(world)]


@pytest.mark.parametrize("world", [2, 3, 4])
def test_layers_with_jitter_are_exact_and_identical(world):
    B, N, layers = 2, 512, 3
    fab = LoopbackFabric(world, 2, B, N)
    parts = [[_parts(world, B, N, 10 * l + j) for j in range(2)] for l in range(layers)]
    x0 = np.random.default_rng(99).standard_normal((B, N)).astype(np.float32)

    def rank_fn(r, rng):
        x = x0.copy()
        for l in range(layers):
            for j in range(2):  # attention output (buffer 0), FFN down (buffer 1)
                fab.push_allreduce(r, j, parts[l][j][r], x, jitter_s=0.002, rng=rng)
        return x

    xs = run_ranks(fab, rank_fn, seed=world)
    want = x0.copy()
    for l in range(layers):
        for j in range(2):
            s = np.zeros((B, N), np.float32)
            for q in range(world):
                s += parts[l][j][q]
            want += s
    for x in xs:
        assert np.array_equal(x.view(np.uint32), xs[0].view(np.uint32))  # bit-identical replicas
        assert np.array_equal(x, want)
    assert fab.err == [0] * world and all(e == [layers, layers] for e in fab.epoch)


def test_silent_rank_times_out_and_epochs_stay_aligned():
    world, B, N = 3, 1, 256
    fab = LoopbackFabric(world, 1, B, N)
    p1, p2 = _parts(world, B, N, 1), _parts(world, B, N, 2)

    def rank_fn(r, rng):
        x = np.zeros((B, N), np.float32)
        # the silent rank waits longer: its peers' later tiles only come after their own timeouts
        fab.push_allreduce(r, 0, p1[r], x, wait_s=0.2 if r != 2 else 3.0, skip_signal=(r == 2))
        after1 = x.copy()
        err1 = fab.err[r]
        fab.err[r] = 0
        fab.push_allreduce(r, 0, p2[r], x, wait_s=2.0)  # next call: everyone aligned again
        return after1, err1, x

    out = run_ranks(fab, rank_fn)
    for r in (0, 1):
        after1, err1, _ = out[r]
        assert err1 == 0x302 and not after1.any()  # waited for rank 2, gave up, x untouched
    s2 = np.zeros((B, N), np.float32)
    for q in range(world):
        s2 += p2[q]
    for r in (0, 1):
        assert np.array_equal(out[r][2], s2)
    # the silent rank itself received everyone's words and completed call 1 without an error, so
    # after a timeout the replicas differ: the host must fail the step on any rank's error word
    assert out[2][1] == 0 and out[2][0].any()
    np.testing.assert_allclose(out[2][2] - out[2][0], s2, rtol=1e-5, atol=1e-3)
    assert all(e == [2] for e in fab.epoch) and fab.err == [0] * world


def test_reuse_without_collective_times_out_instead_of_mixing_epochs():
    world, B, N = 2, 1, 128
    fab = LoopbackFabric(world, 1, B, N)
    pa, pb = _parts(world, B, N, 3), _parts(world, B, N, 4)

    def rank_fn(r, rng):
        x = np.zeros((B, N), np.float32)
        # rank 0 is slow to read: rank 1 finishes call A and overwrites the slot with call B's epoch
        fab.push_allreduce(r, 0, pa[r], x, wait_s=0.5, pause_after_write_s=0.3 if r == 0 else 0.0)
        e = fab.err[r]
        fab.push_allreduce(r, 0, pb[r], x, wait_s=2.0)
        return e, x

    (e0, x0), (e1, x1) = run_ranks(fab, rank_fn)
    assert e0 == 0x301 and e1 == 0  # the slow rank reports a timeout for call A ...
    sb = pb[0] + pb[1]
    assert np.array_equal(x0, sb)  # ... and never added a sum built from mixed epochs
    assert np.array_equal(x1, (pa[0] + pa[1]) + sb)
