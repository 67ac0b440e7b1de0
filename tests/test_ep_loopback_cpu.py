"""CPU model of the expert-parallel all-to-all protocol (parallel/ep_loopback.py): counts exchange,
dispatch into the experts' ranks, expert compute, weighted gather back, several MoE layers back to
back on threads with random delays and no barrier."""
import numpy as np
import pytest

from barq_inference_b200.parallel.ep_loopback import recv_row_base, run_layers


@pytest.mark.parametrize("world,E,k", [(2, 4, 2), (4, 8, 2), (8, 64, 6), (8, 8, 2)])
def test_all_to_all_layers_match_reference(world, E, k):
    for seed in range(2):
        got, ref = run_layers(world, E, k, rows=5, H=32, layers=3, seed=seed)
        for a, b in zip(got, ref):
            assert np.allclose(a, b, rtol=1e-5, atol=1e-5), np.abs(a - b).max()


def test_receive_layout_is_expert_major_then_source_rank():
    cm = np.array([[1, 2, 0, 3],   # rank 0's rows per expert
                   [4, 0, 5, 1]])  # rank 1's
    # two experts per rank: owner 0 holds experts 0, 1; owner 1 holds 2, 3
    assert recv_row_base(cm, 2, 0, 0) == 0 and recv_row_base(cm, 2, 0, 1) == 1
    assert recv_row_base(cm, 2, 1, 0) == 5 and recv_row_base(cm, 2, 1, 1) == 7
    assert recv_row_base(cm, 2, 2, 0) == 0 and recv_row_base(cm, 2, 3, 1) == 5 + 3
