"""TQ1_0 / TQ2_0 ternary GGUF types: hand-built known vectors, quantize round trip, lossless Q4_0
import, GGUF file round trip (CPU)."""
import numpy as np
import torch

from barq_inference_b200.gguf import GGMLType, GGUFWriter, dequantize, quantize, read_gguf
from barq_inference_b200.gguf.ternary import to_q4_0


def test_tq2_0_known_bytes():
    b = np.zeros(66, np.uint8)
    b[0] = 0b10_01_00_10  # values 0, 32, 64, 96 -> codes 2, 0, 1, 2
    b[33] = 0b00_00_00_00  # group 1, m=1: values 129, 161, 193, 225 -> code 0 (-d)
    b[64:66] = np.array([0.5], np.float16).view(np.uint8)
    y = dequantize(b, GGMLType.TQ2_0)
    assert (y[0], y[32], y[64], y[96]) == (0.5, -0.5, 0.0, 0.5)
    assert (y[129], y[161], y[193], y[225]) == (-0.5, -0.5, -0.5, -0.5)


def test_tq1_0_known_bytes():
    b = np.zeros(54, np.uint8)
    b[:52] = 0x80  # digits of 128: (1, 1, 1, 1, 1) as a base-3 fraction -> code 1 (zero) ... check below
    digits = (2, 0, 1, 1, 0)
    v = sum(t * 3 ** (4 - i) for i, t in enumerate(digits))
    b[0] = -(-v * 256 // 243)  # ceil(v * 256 / 243)
    b[52:54] = np.array([2.0], np.float16).view(np.uint8)
    y = dequantize(b, GGMLType.TQ1_0)
    assert [y[n * 32] for n in range(5)] == [2.0 * (t - 1) for t in digits]  # byte 0 holds values n*32


def test_quantize_roundtrip_and_q4_0_import(tmp_path):
    x = torch.randn(8, 512)
    for t in (GGMLType.TQ1_0, GGMLType.TQ2_0):
        q = quantize(x, t).numpy()
        y = dequantize(q, t, (8, 512)).reshape(-1, 256)
        d = np.abs(x.numpy()).reshape(-1, 256).max(1).astype(np.float16).astype(np.float32)
        want = np.clip(np.rint(x.numpy().reshape(-1, 256) / np.abs(x.numpy()).reshape(-1, 256).max(1, keepdims=True)),
                       -1, 1) * d[:, None]
        assert np.array_equal(y, want)
        assert np.array_equal(dequantize(to_q4_0(q, t == GGMLType.TQ1_0), GGMLType.Q4_0), y.reshape(-1))
        p = tmp_path / f"{t.name}.gguf"
        w = GGUFWriter(p, arch="llama")
        w.add_tensor("w", q, t, (8, 512))
        w.write()
        g = read_gguf(p)
        assert g.tensor("w").ggml_type == t and np.array_equal(g.tensor("w").rows().reshape(-1), q.reshape(-1))
        from barq_inference_b200.models.weights import tensors_from_gguf

        pt = tensors_from_gguf(g)["w"]
        assert pt.ggml_type == GGMLType.Q4_0
        assert np.array_equal(dequantize(pt.data.numpy(), GGMLType.Q4_0, (8, 512)).reshape(-1, 256), y)
