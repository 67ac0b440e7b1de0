"""Import of block types without a kernel format: Q3_K as Q6_K rows (exact), IQ4_XS as IQ4_NL rows
(block scales rounded to fp16), Q5_0, Q2_K, Q4_1, Q5_1 as Q8_0 rows.

Q3_K maps exactly onto Q6_K (same super-block, signed sub-block scales, codes shifted by 32) and Q5_0
onto Q8_0 (same block size and scale); the others are requantized with an error of about one Q8_0
step (1/254 of each 32-value block's largest magnitude, plus the fp16 rounding of its scale).
Random block bytes with a fixed, finite fp16 scale are valid blocks of every type."""
import numpy as np
import pytest
import torch

from barq_inference_b200.gguf import GGMLType, dequantize, quantize
from barq_inference_b200.ops.qweight import W_BF16, QWeight, iq4_xs_as_iq4_nl, q3_k_as_q6_k, requant_q8_0

N, K = 8, 512
LAYOUT = {GGMLType.Q3_K: (256, 110, [108]), GGMLType.IQ4_XS: (256, 136, [0]), GGMLType.Q2_K: (256, 84, [80, 82]),
          GGMLType.Q4_1: (32, 20, [0, 2]), GGMLType.Q5_1: (32, 24, [0, 2]), GGMLType.Q5_0: (32, 22, [0])}


def _random_blocks(t, seed=0):
    qk, bs, doffs = LAYOUT[t]
    raw = np.random.default_rng(seed).integers(0, 256, (N, K // qk, bs), dtype=np.uint8)
    for o in doffs:
        raw[..., o:o + 2] = np.frombuffer(np.float16(0.01).tobytes(), np.uint8)
    return torch.from_numpy(raw.reshape(N, -1).copy())


def test_q5_0_is_exact():
    w = torch.randn(N, K, generator=torch.Generator().manual_seed(1))
    raw = quantize(w, GGMLType.Q5_0)
    q8 = requant_q8_0(raw, GGMLType.Q5_0, N, K)
    assert np.array_equal(dequantize(q8.numpy(), GGMLType.Q8_0, (N, K)), dequantize(raw.numpy(), GGMLType.Q5_0, (N, K)))
    assert np.array_equal(dequantize(requant_q8_0(_random_blocks(GGMLType.Q5_0), GGMLType.Q5_0, N, K).numpy(),
                                     GGMLType.Q8_0, (N, K)),
                          dequantize(_random_blocks(GGMLType.Q5_0).numpy(), GGMLType.Q5_0, (N, K)))


@pytest.mark.parametrize("t", [GGMLType.Q3_K, GGMLType.Q2_K, GGMLType.Q4_1, GGMLType.Q5_1])
def test_requantized_within_one_q8_step(t):
    raw = _random_blocks(t)
    ref = dequantize(raw.numpy(), t, (N, K))
    got = dequantize(requant_q8_0(raw, t, N, K).numpy(), GGMLType.Q8_0, (N, K))
    # half a Q8_0 step (max/254) plus the fp16 rounding of the scale (127 steps x 2^-11 of a step)
    bound = np.abs(ref.reshape(N, -1, 32)).max(-1, keepdims=True) / 220
    assert (np.abs(got - ref).reshape(N, -1, 32) <= bound).all()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_q3_k_is_exact_as_q6_k(seed):
    raw = _random_blocks(GGMLType.Q3_K, seed)
    raw.view(N, -1, 110)[..., 108:110] = torch.from_numpy(  # a different fp16 scale per block
        np.random.default_rng(seed).uniform(1e-3, 0.5, (N, K // 256)).astype(np.float16).view(np.uint8).reshape(N, -1, 2))
    q6 = q3_k_as_q6_k(raw, N, K)
    assert q6.shape == (N, K // 256 * 210) and q6.dtype == torch.uint8
    assert np.array_equal(dequantize(q6.numpy(), GGMLType.Q6_K, (N, K)), dequantize(raw.numpy(), GGMLType.Q3_K, (N, K)))
    try:  # the C++ oracle the device kernels are checked against reads the Q6_K rows the same way
        from barq_inference_b200 import _cpu_ref
    except ImportError:
        _cpu_ref = None
    if _cpu_ref is not None:
        got = _cpu_ref.dequantize(q6.reshape(-1).contiguous(), int(GGMLType.Q6_K), N * K).numpy()
        assert np.array_equal(got.reshape(N, K), dequantize(raw.numpy(), GGMLType.Q3_K, (N, K)))
    # the loader streams Q3_K as exactly these Q6_K rows
    w = QWeight.from_packed(raw, GGMLType.Q3_K, N, K, "cpu")
    assert w.wtype == int(GGMLType.Q6_K)
    assert torch.equal(w.to_gguf_rows().cpu(), q6)


@pytest.mark.parametrize("seed", [0, 1])
def test_iq4_xs_as_iq4_nl_rounds_only_the_block_scales(seed):
    raw = _random_blocks(GGMLType.IQ4_XS, seed)
    raw.view(N, -1, 136)[..., 0:2] = torch.from_numpy(
        np.random.default_rng(seed).uniform(1e-3, 0.05, (N, K // 256)).astype(np.float16).view(np.uint8).reshape(N, -1, 2))
    nl = iq4_xs_as_iq4_nl(raw, N, K)
    assert nl.shape == (N, K // 32 * 18)
    ref = dequantize(raw.numpy(), GGMLType.IQ4_XS, (N, K))
    got = dequantize(nl.numpy(), GGMLType.IQ4_NL, (N, K))
    assert (np.abs(got - ref) <= np.abs(ref) * 2.0 ** -11 + 1e-12).all()  # half an fp16 ulp of the scale
    # codes are untouched: dividing out each block's scale gives the same codebook values
    dxs = dequantize(raw.numpy(), GGMLType.IQ4_XS, (N, K)).reshape(N, -1, 32)
    assert np.array_equal(np.sign(got.reshape(N, -1, 32)), np.sign(dxs))
    assert QWeight.from_packed(raw, GGMLType.IQ4_XS, N, K, "cpu").wtype == int(GGMLType.IQ4_NL)
    try:  # the C++ oracle of the device kernels reads the converted rows as the Python oracle does
        from barq_inference_b200 import _cpu_ref
    except ImportError:
        _cpu_ref = None
    if _cpu_ref is not None:
        c = _cpu_ref.dequantize(nl.reshape(-1).contiguous(), int(GGMLType.IQ4_NL), N * K).numpy().reshape(N, K)
        assert np.array_equal(c, got)


def test_loader_streams_requantized_types():
    w = QWeight.from_packed(_random_blocks(GGMLType.Q2_K), GGMLType.Q2_K, N, K, "cpu")
    assert w.wtype == int(GGMLType.Q8_0) and w.wtype != W_BF16
    w = QWeight.from_packed(_random_blocks(GGMLType.Q3_K), GGMLType.Q3_K, N, K, "cpu")
    assert w.wtype == int(GGMLType.Q6_K)
