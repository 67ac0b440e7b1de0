"""GGUF format and ggml block layouts (CPU)."""
import numpy as np
import pytest
import torch

from barq_inference_b200.gguf import (GGMLType, GGUFWriter, GGUFValueType, QUANTIZERS, TYPE_TRAITS, dequantize,
                                      quantize, read_gguf, read_gguf_bytes, GGUFError)


def test_roundtrip_metadata_and_tensors(tmp_path):
    p = tmp_path / "t.gguf"
    w = GGUFWriter(p, arch="llama")
    w.add("llama.block_count", 2)
    w.add("f", 1.5)
    w.add("neg", -3)
    w.add("s", "héllo")
    w.add("b", True)
    w.add("arr_s", ["a", "bb", "ccc"])
    w.add("arr_i", [1, 2, 3])
    w.add("arr_f", np.array([0.5, 1.5], np.float32))
    w.add("nested", [[1, 2], [3]], GGUFValueType.ARRAY, GGUFValueType.ARRAY)
    w.add("u64", 2**40, GGUFValueType.UINT64)
    x = torch.randn(8, 256)
    q = quantize(x, GGMLType.Q4_K)
    w.add_tensor("w", q.numpy(), GGMLType.Q4_K, (8, 256))
    w.add_tensor("n", np.ones(256, np.float32), GGMLType.F32, (256,))
    w.write()
    g = read_gguf(p)
    assert g.version == 3 and g.architecture == "llama"
    assert g.get("llama.block_count") == 2 and g.get("neg") == -3 and g.get("s") == "héllo"
    assert g.get("b") is True and g.get("arr_s") == ["a", "bb", "ccc"] and g.get("arr_i") == [1, 2, 3]
    assert g.get("nested") == [[1, 2], [3]] and g.get("u64") == 2**40
    assert abs(g.get("f") - 1.5) < 1e-9
    t = g.tensor("w")
    assert t.shape == (256, 8) and t.torch_shape == (8, 256) and t.ggml_type == GGMLType.Q4_K
    assert np.array_equal(t.rows(), q.numpy())
    assert g.data_offset % 32 == 0 and (g.data_offset + t.offset) % 32 == 0


def test_bad_files():
    with pytest.raises(GGUFError):
        read_gguf_bytes(b"XXXX" + b"\0" * 40)
    with pytest.raises(GGUFError):
        read_gguf_bytes(b"GGUF" + (3).to_bytes(4, "little") + (5).to_bytes(8, "little"))


@pytest.mark.parametrize("t", [t for t in QUANTIZERS if TYPE_TRAITS[t].block_size > 1])
def test_quant_roundtrip_error(t):
    torch.manual_seed(0)
    x = torch.randn(16, 512) * 0.02
    y = dequantize(quantize(x, t).numpy(), t, (16, 512))
    bits = TYPE_TRAITS[t].type_size * 8 / TYPE_TRAITS[t].block_size
    rel = np.abs(y - x.numpy()).max() / np.abs(x.numpy()).max()
    assert rel < 2.0 ** (-bits + 2.3), (t, rel)


def test_known_vectors_q4_0_q8_0():
    # hand-built ggml blocks: Q4_0 d=0.5, nibble j = j % 16  -> x[j] = (j%16 - 8) * 0.5
    d = np.array([0.5], np.float16).view(np.uint8)
    qs = np.array([(j % 16) | ((15 - j % 16) << 4) for j in range(16)], np.uint8)
    blk = np.concatenate([d, qs])
    y = dequantize(blk, GGMLType.Q4_0)
    assert y[3] == (3 - 8) * 0.5 and y[16 + 3] == (12 - 8) * 0.5
    d8 = np.array([0.25], np.float16).view(np.uint8)
    q8 = np.arange(-16, 16, dtype=np.int8).view(np.uint8)
    y8 = dequantize(np.concatenate([d8, q8]), GGMLType.Q8_0)
    assert np.array_equal(y8, np.arange(-16, 16) * 0.25)


def test_known_vector_q4_k_scales():
    # one Q4_K block: d=1, dmin=0.5, sub-block j scale=j+1 min=j, all nibbles 3
    sc = np.zeros(12, np.uint8)
    ls, lm = list(range(1, 9)), list(range(8))
    for j in range(4):
        sc[j] = ls[j] | ((ls[j + 4] >> 4) << 6)
        sc[j + 4] = lm[j] | ((lm[j + 4] >> 4) << 6)
        sc[j + 8] = (ls[j + 4] & 0xF) | ((lm[j + 4] & 0xF) << 4)
    blk = np.concatenate([np.array([1.0, 0.5], np.float16).view(np.uint8), sc, np.full(128, 0x33, np.uint8)])
    y = dequantize(blk, GGMLType.Q4_K)
    for j in range(8):
        assert np.allclose(y[32 * j:32 * j + 32], (j + 1) * 3 - 0.5 * j)


def test_iq4_nl_codebook():
    d = np.array([1.0], np.float16).view(np.uint8)
    qs = np.array([(j) | ((15 - j) << 4) for j in range(16)], np.uint8)
    y = dequantize(np.concatenate([d, qs]), GGMLType.IQ4_NL)
    assert y[0] == -127 and y[15] == 113 and y[16] == 113 and y[31] == -127


def test_cpu_ref_matches_numpy():
    from barq_inference_b200 import _cpu_ref

    torch.manual_seed(1)
    x = torch.randn(4, 512) * 0.02
    for t in (GGMLType.Q4_0, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q5_K, GGMLType.Q6_K, GGMLType.IQ4_NL):
        raw = quantize(x, t)
        a = _cpu_ref.dequantize(raw.reshape(-1).contiguous(), int(t), 4 * 512).numpy()
        b = dequantize(raw.numpy(), t)
        assert np.array_equal(a, b), t
        v = torch.randn(2, 512)
        y = _cpu_ref.qgemv(raw.reshape(-1).contiguous(), int(t), 4, 512, v)
        assert torch.allclose(y, v @ torch.from_numpy(b.reshape(4, 512)).T, atol=1e-5)


def test_split_gguf_roundtrip(tmp_path):
    """gguf-split layout: 3 parts, metadata in the first, tensors merged on read."""
    from barq_inference_b200.gguf import read_gguf_split, split_paths
    from barq_inference_b200.models import POLICIES, preset, random_tensors
    from barq_inference_b200.models.weights import tensors_from_gguf, write_gguf_split

    cfg = preset("tiny")
    t = random_tensors(cfg, POLICIES["tiny"], seed=2)
    parts = write_gguf_split(str(tmp_path / "m.gguf"), cfg, t, 3)
    assert split_paths(parts[1]) == parts
    g = read_gguf_split(parts[0])
    assert g.metadata["split.count"] == 3 and g.architecture == "llama"
    back = tensors_from_gguf(g)
    assert set(back) == set(t)
    for k in t:
        assert torch.equal(back[k].data, t[k].data), k
    # opening any part finds the whole model
    assert set(read_gguf_split(parts[2]).tensors) == set(t)
