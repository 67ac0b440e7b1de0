"""ik_llama row-scaled quant types, the Q4_K_R4 repack and the IKQ1 archive (CPU)."""
import struct

import numpy as np
import pytest
import torch

from barq_inference_b200.gguf import GGMLType, GGUFWriter, dequantize, quantize, read_gguf, row_nbytes
from barq_inference_b200.gguf.constants import KVALUES_IQ2NL, KVALUES_IQ3NL, KVALUES_IQ4K
from barq_inference_b200.gguf.ik_quants import repack_q4_k_r4, unpack_q4_k_r4
from barq_inference_b200.gguf.ikq import IKQ_Q4_K_R4, IKQ_RAW, gguf_to_ikq, ikq_to_gguf, read_ikq

IK = [GGMLType.IQ4_KS, GGMLType.IQ3_KS, GGMLType.IQ2_KS]


def test_row_sizes():
    assert row_nbytes(GGMLType.IQ4_KS, 512) == 4 + 2 * 136
    assert row_nbytes(GGMLType.IQ3_KS, 256) == 2 + 102
    assert row_nbytes(GGMLType.IQ2_KS, 4096) == 2 + 16 * 70


def test_known_vector_iq4_ks():
    d = np.array([0.5], "<f4").view(np.uint8)
    # byte = (level + 127) | half: level +3 shifted, level -3 base, then level +1 base
    scales = np.array([130 | 1, 124] + [128] * 6, np.uint8)
    qs = np.zeros(128, np.uint8)
    qs[0:16] = np.arange(16) | ((15 - np.arange(16)) << 4)
    qs[16:32] = 0x21
    row = np.concatenate([d, scales, qs])
    y = dequantize(row, GGMLType.IQ4_KS, (1, 256))[0]
    v = np.array(KVALUES_IQ4K, np.float32)
    lvl0 = (int(scales[0]) & 254) - 127
    assert lvl0 == 3
    assert np.allclose(y[0:16], 0.5 * lvl0 * v[16 + np.arange(16)])
    assert np.allclose(y[16:32], 0.5 * lvl0 * v[16 + 15 - np.arange(16)])
    lvl1 = (int(scales[1]) & 254) - 127
    assert np.allclose(y[32:48], 0.5 * lvl1 * v[1]) and np.allclose(y[48:64], 0.5 * lvl1 * v[2])


def test_known_vector_iq2_ks():
    d = np.array([0.25], np.float16).view(np.uint8)
    # block 0: scale nibble 5, high bit 1 (extra bit 8) -> ls 21 -> 5; shifted (extra bit 0)
    # block 5: scale nibble 0 (high nibble of scales[2]), high bit 0 -> -16; base values
    extra = (1 << 8) | 1
    scales = np.array([5, 0, 0x00, 0], np.uint8)
    qs = np.zeros(64, np.uint8)
    qs[0:32] = np.arange(32) % 4  # block 0: bits 0-1
    qs[32:64] = (np.arange(32) % 4) << 2  # block 5 = 4 + 1: second half of qs, shift 2
    blk = np.concatenate([np.array([extra], "<u2").view(np.uint8), scales, qs])
    y = dequantize(np.concatenate([d, blk]), GGMLType.IQ2_KS, (1, 256))[0]
    v = np.array(KVALUES_IQ2NL, np.float32)
    assert np.allclose(y[0:32], 0.25 * 5 * v[4 + np.arange(32) % 4])
    assert np.allclose(y[160:192], 0.25 * -16 * v[np.arange(32) % 4])


def test_known_vector_iq3_ks():
    d = np.array([0.125], np.float16).view(np.uint8)
    # block 6 (second 128, ib 2): scale nibble = high nibble of scales[2]; high bit = extra bit 6;
    # codebook half = extra bit 14; low 2 bits at qs[32 + j] >> 4; bit 2 from qh[j] >> 6
    extra = (1 << 6) | (1 << 14)
    scales = np.array([0, 0, 0x70, 0], np.uint8)  # nibble 7 | 16 -> 23 -> +7
    qs = np.zeros(64, np.uint8)
    qs[32:64] = (np.arange(32) % 4) << 4
    qh = ((np.arange(32) // 4 % 2) << 6).astype(np.uint8)
    blk = np.concatenate([np.array([extra], "<u2").view(np.uint8), scales, qs, qh])
    y = dequantize(np.concatenate([d, blk]), GGMLType.IQ3_KS, (1, 256))[0]
    v = np.array(KVALUES_IQ3NL, np.float32)
    j = np.arange(32)
    assert np.allclose(y[192:224], 0.125 * 7 * v[8 + ((j % 4) | ((j // 4 % 2) << 2))])
    assert np.allclose(y[0:32], 0.125 * -16 * v[0])  # block 0: all-zero fields -> level -16, code 0


@pytest.mark.parametrize("t,bound", [(GGMLType.IQ4_KS, 0.09), (GGMLType.IQ3_KS, 0.17), (GGMLType.IQ2_KS, 0.34)])
def test_quantize_roundtrip_rms(t, bound):
    torch.manual_seed(0)
    x = torch.randn(16, 1024) * 0.03
    q = quantize(x, t)
    assert q.shape == (16, row_nbytes(t, 1024))
    y = dequantize(q.numpy(), t, (16, 1024))
    rel = np.sqrt(((y - x.numpy()) ** 2).mean()) / x.numpy().std()
    assert rel < bound, rel


def test_q4_k_r4_repack_is_lossless():
    x = torch.randn(12, 512)
    q = quantize(x, GGMLType.Q4_K).numpy()
    p = repack_q4_k_r4(q)
    assert p.shape == (3, 2 * 576)
    assert np.array_equal(unpack_q4_k_r4(p, 12), q)
    with pytest.raises(ValueError):
        repack_q4_k_r4(q[:6])


def _tiny_gguf(path, t=GGMLType.Q8_0):
    torch.manual_seed(1)
    w = GGUFWriter(path, arch="llama")
    w.add("llama.block_count", 1)
    w.add("tokenizer.ggml.tokens", ["a", "b"])
    mats = {"blk.0.ffn_up.weight": torch.randn(8, 512) * 0.02, "blk.0.attn_q.weight": torch.randn(4, 256)}
    for n, m in mats.items():
        w.add_tensor(n, quantize(m, t).numpy(), t, tuple(m.shape))
    w.add_tensor("blk.0.attn_norm.weight", np.linspace(0.5, 1.5, 256).astype(np.float32), GGMLType.F32, (256,))
    w.write()
    return read_gguf(path)


@pytest.mark.parametrize("t", IK)
def test_gguf_with_ik_tensors_reads_and_imports(tmp_path, t):
    from barq_inference_b200.gguf.ik_quants import import_type
    from barq_inference_b200.models.weights import tensors_from_gguf

    x = torch.randn(8, 512) * 0.02
    w = GGUFWriter(tmp_path / "ik.gguf", arch="llama")
    w.add_tensor("w", quantize(x, t).numpy(), t, (8, 512))
    w.write()
    g = read_gguf(tmp_path / "ik.gguf")
    ti = g.tensor("w")
    assert ti.ggml_type == t and ti.rows().shape == (8, row_nbytes(t, 512))
    ref = dequantize(ti.rows(), t, (8, 512))
    pt = tensors_from_gguf(g)["w"]
    assert pt.ggml_type == import_type(t)
    got = dequantize(pt.data.numpy(), pt.ggml_type, (8, 512))
    assert np.abs(got - ref).max() <= 0.1 * np.abs(ref).max()


@pytest.mark.parametrize("quant", ["iq4_ks", "q4_k_r4"])
def test_ikq_archive_roundtrip(tmp_path, quant):
    g = _tiny_gguf(tmp_path / "m.gguf")
    gguf_to_ikq(str(tmp_path / "m.gguf"), str(tmp_path / "m.ikq"), quant, device="cpu")
    raw = open(tmp_path / "m.ikq", "rb").read()
    assert raw[:4] == b"IKQ1" and struct.unpack("<III", raw[4:16])[0] == 1
    a = read_ikq(str(tmp_path / "m.ikq"))
    assert a.metadata["llama.block_count"] == 1 and a.metadata["ik.quant_type"] == quant
    assert a.tensors["blk.0.attn_norm.weight"].quant == IKQ_RAW
    assert a.tensors["blk.0.ffn_up.weight"].shape == (8, 512)
    if quant == "q4_k_r4":
        assert a.tensors["blk.0.ffn_up.weight"].quant == IKQ_Q4_K_R4
        assert a.tensors["blk.0.ffn_up.weight"].data.size == 2 * 2 * 576
    ikq_to_gguf(str(tmp_path / "m.ikq"), str(tmp_path / "back.gguf"))
    b = read_gguf(tmp_path / "back.gguf")
    assert b.get("tokenizer.ggml.tokens") == ["a", "b"] and b.get("llama.block_count") == 1
    for name, ti in g.tensors.items():
        ref = dequantize(np.array(ti.data), ti.ggml_type, ti.torch_shape)
        bt = b.tensor(name)
        got = dequantize(np.array(bt.data), bt.ggml_type, bt.torch_shape)
        assert np.abs(got - ref).max() <= 0.15 * np.abs(ref).max(), name
    assert np.array_equal(np.array(b.tensor("blk.0.attn_norm.weight").data).view("<f4"),
                          np.linspace(0.5, 1.5, 256).astype(np.float32))


def test_cli_convert_to_ik_gguf(tmp_path):
    from barq_inference_b200.cli import main

    _tiny_gguf(tmp_path / "m.gguf")
    assert main(["convert", "--input", str(tmp_path / "m.gguf"), "--output", str(tmp_path / "o.gguf"),
                 "--quantize", "iq3_ks", "--device", "cpu"]) == 0
    o = read_gguf(tmp_path / "o.gguf")
    assert o.tensor("blk.0.ffn_up.weight").ggml_type == GGMLType.IQ3_KS
    assert o.tensor("blk.0.attn_norm.weight").ggml_type == GGMLType.F32
