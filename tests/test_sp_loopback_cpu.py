"""CPU model of the sequence-parallel reduce-scatter / all-gather protocol (parallel/sp_loopback.py):
ranks as threads with random delays and random tile order inside every kernel.  Reusing the receive
slots and gather buffers from layer to layer without barriers must never read a stale or
overwritten row, and the residual stream must match the sequential reference."""
import numpy as np
import pytest

from barq_inference_b200.parallel.sp_loopback import ProtocolError, SpFabric, run_layers


@pytest.mark.parametrize("world,T", [(2, 10), (3, 7), (4, 16), (8, 9)])
def test_layers_without_barriers_match_reference(world, T):
    for seed in range(3):
        xs, ref = run_layers(world, T, 256, layers=3, seed=seed)
        got = np.concatenate([x for x in xs if len(x)])
        assert got.shape == ref.shape
        assert np.allclose(got, ref, rtol=1e-4, atol=1e-4), np.abs(got - ref).max()


def test_a_slot_overwritten_early_is_caught():
    """A rank that pushes its next call's tiles before the owner consumed the current ones (what
    the data dependencies rule out) is detected by the epoch tags, not silently summed."""
    fab = SpFabric(2, 8, 128, bn=4)
    part = np.ones((8, 128), np.float32)
    fab.gemm_rs(1, 0, part)                # call 1 of rank 1
    fab.epoch[1][0] += 1                   # rank 1 runs ahead ...
    fab.gemm_rs(1, 0, part)                # ... and overwrites the owner's slots with call 2
    fab.gemm_rs(0, 0, part)
    with pytest.raises(ProtocolError):
        fab.reduce_norm_ag(0, 0, np.zeros((4, 128), np.float32), np.ones(128, np.float32))
