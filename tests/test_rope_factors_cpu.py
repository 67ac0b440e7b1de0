"""Per-dimension RoPE frequency factors (GGUF rope_freqs.weight) and LongRoPE tables (CPU)."""
import dataclasses
import math

import numpy as np
import torch

from barq_inference_b200.gguf import GGMLType, GGUFWriter, read_gguf
from barq_inference_b200.models import preset
from barq_inference_b200.models.config import attach_rope_factors
from barq_inference_b200.models.rope import rope_cos_sin


def _expected(d, base, ff, n, mscale):
    inv = np.array([1.0 / (base ** (2 * i / d) * ff[i]) for i in range(d // 2)])
    th = np.arange(n)[:, None] * inv[None]
    return np.cos(th) * mscale, np.sin(th) * mscale


def test_freq_factors_divide_inverse_frequencies():
    cfg = preset("tiny")
    d = cfg.rot_dim
    ff = tuple(1.0 + 0.25 * i for i in range(d // 2))
    c = dataclasses.replace(cfg, rope_freq_factors=ff)
    cos, sin = rope_cos_sin(c, 64)
    ec, es = _expected(d, c.rope_theta, ff, 64, 1.0)
    assert np.allclose(cos.numpy(), ec, atol=1e-6) and np.allclose(sin.numpy(), es, atol=1e-6)


def test_longrope_attention_factor():
    cfg = dataclasses.replace(preset("tiny"), max_ctx=16384, rope_orig_ctx=4096, rope_scaling="longrope")
    d = cfg.rot_dim
    ff = tuple(1.0 + 0.1 * i for i in range(d // 2))
    c = dataclasses.replace(cfg, rope_freq_factors=ff)
    cos, _ = rope_cos_sin(c, 32)
    m = math.sqrt(1 + math.log(4.0) / math.log(4096))
    ec, _ = _expected(d, c.rope_theta, ff, 32, m)
    assert np.allclose(cos.numpy(), ec, atol=1e-6)
    c2 = dataclasses.replace(c, rope_attn_factor=1.5)
    assert abs(float(rope_cos_sin(c2, 1)[0][0, 0]) - 1.5) < 1e-6


def test_attach_from_gguf(tmp_path):
    cfg = dataclasses.replace(preset("tiny"), max_ctx=8192, rope_orig_ctx=4096)
    d2 = cfg.rot_dim // 2
    p = tmp_path / "r.gguf"
    w = GGUFWriter(p, arch="llama")
    w.add_tensor("rope_factors_long.weight", np.full(d2, 2.0, np.float32), GGMLType.F32, (d2,))
    w.add_tensor("rope_factors_short.weight", np.full(d2, 1.0, np.float32), GGMLType.F32, (d2,))
    w.write()
    g = read_gguf(p)
    c = attach_rope_factors(dataclasses.replace(cfg), g)
    assert c.rope_scaling == "longrope" and c.rope_freq_factors == (2.0,) * d2  # 8192 > 4096: long
    c = attach_rope_factors(dataclasses.replace(cfg, max_ctx=4096), g)
    assert c.rope_freq_factors == (1.0,) * d2
    p2 = tmp_path / "f.gguf"
    w = GGUFWriter(p2, arch="llama")
    w.add_tensor("rope_freqs.weight", np.arange(1, d2 + 1, dtype=np.float32), GGMLType.F32, (d2,))
    w.write()
    c = attach_rope_factors(dataclasses.replace(cfg), read_gguf(p2))
    assert c.rope_scaling == "none" and c.rope_freq_factors[-1] == float(d2)
    torch.testing.assert_close(rope_cos_sin(c, 4)[0][1, 1], torch.tensor(math.cos(1 / (cfg.rope_theta ** (2 / cfg.rot_dim) * 2))),
                               atol=1e-6, rtol=0)
