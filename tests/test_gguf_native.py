"""Native (C++) GGUF parser == the Python parser: every metadata value type, long numeric arrays,
tensor views, and fuzzed (truncated / byte-flipped) headers, which must fail cleanly in both."""
import numpy as np
import pytest
import torch

from barq_inference_b200.gguf import GGMLType, GGUFValueType, GGUFWriter, quantize, read_gguf

nat = pytest.importorskip("barq_inference_b200._native")


def _fixture(path):
    w = GGUFWriter(path, arch="llama")
    w.add("llama.block_count", 2)
    w.add("f", 1.5)
    w.add("neg", -3)
    w.add("s", "héllo")
    w.add("b", True)
    w.add("arr_s", ["a", "bb", "ccc"])
    w.add("arr_i", [1, 2, 3])
    w.add("arr_f", np.array([0.5, 1.5], np.float32))
    w.add("long_f", np.arange(1000, dtype=np.float32))
    w.add("long_i64", np.arange(100, dtype=np.int64) - 50)
    w.add("nested", [[1, 2], [3]], GGUFValueType.ARRAY, GGUFValueType.ARRAY)
    w.add("u64", 2**40, GGUFValueType.UINT64)
    w.add("i8", -5, GGUFValueType.INT8)
    w.add("u16", 60000, GGUFValueType.UINT16)
    w.add("f64", 2.25, GGUFValueType.FLOAT64)
    x = torch.randn(8, 256, generator=torch.Generator().manual_seed(0))
    w.add_tensor("w", quantize(x, GGMLType.Q4_K).numpy(), GGMLType.Q4_K, (8, 256))
    w.add_tensor("n", np.ones(256, np.float32), GGMLType.F32, (256,))
    w.write()


def _same(a, b):
    assert a.version == b.version and a.alignment == b.alignment and a.data_offset == b.data_offset
    assert a.metadata.keys() == b.metadata.keys() and a.metadata_types == b.metadata_types
    for k, v in a.metadata.items():
        u = b.metadata[k]
        if isinstance(v, np.ndarray):
            assert isinstance(u, np.ndarray) and v.dtype == u.dtype and np.array_equal(v, u), k
        else:
            assert v == u and type(v) is type(u), k
    assert a.tensors.keys() == b.tensors.keys()
    for k, t in a.tensors.items():
        s = b.tensors[k]
        assert (t.shape, t.ggml_type, t.offset) == (s.shape, s.ggml_type, s.offset)
        assert np.array_equal(t.data, s.data)


def test_native_matches_python(tmp_path):
    p = tmp_path / "t.gguf"
    _fixture(p)
    a, b = read_gguf(p, native=True), read_gguf(p, native=False)
    _same(a, b)
    assert not a.tensors["w"].data.flags.writeable  # read-only mapping
    del b
    a.close()


def test_native_fuzzed_headers_fail_like_python(tmp_path):
    p = tmp_path / "t.gguf"
    _fixture(p)
    raw = p.read_bytes()
    rng = np.random.default_rng(0)
    head_len = read_gguf(p, native=False).data_offset
    cases = [raw[:n] for n in (24, 30, 64, head_len // 2, head_len - 1)]
    for _ in range(400):
        b = bytearray(raw)
        for _ in range(int(rng.integers(1, 4))):
            b[int(rng.integers(0, head_len))] = int(rng.integers(0, 256))
        cases.append(bytes(b))
    q = tmp_path / "f.gguf"
    n_ok = 0
    for c in cases:
        q.write_bytes(c)
        res = []
        for native in (True, False):
            try:
                res.append(read_gguf(q, native=native))
            except (ValueError, OverflowError, MemoryError, ZeroDivisionError):
                res.append(None)
        a, b = res
        assert (a is None) == (b is None)
        if a is not None:
            _same(a, b)
            n_ok += 1
    assert n_ok < len(cases)  # most corruptions are caught
