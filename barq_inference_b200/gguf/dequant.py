"""ggml-spec block dequantization in NumPy: the CPU correctness oracle.

Written from the public ggml block definitions.  The reference's K-quant dequantizers
(``barq_core/src/gguf.rs:635-1208``) agree with ggml; its Q4_0 reader (``gguf.rs:522-578``)
does not (f32 scale, interleaved nibbles) and is deliberately not followed.

Every function takes the packed bytes (any shape whose size is a multiple of the block
size in bytes) and returns ``float32`` values with one row per block.
"""
from __future__ import annotations

import numpy as np

from .constants import KVALUES_IQ4NL, QK_K, TYPE_TRAITS, GGMLType


def _blocks(raw: np.ndarray, t: GGMLType) -> np.ndarray:
    ts = TYPE_TRAITS[t].type_size
    b = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
    if b.size % ts:
        raise ValueError(f"{t.name}: {b.size} bytes is not a whole number of {ts}-byte blocks")
    return b.reshape(-1, ts)


def _f16(b: np.ndarray, off: int) -> np.ndarray:
    return b[:, off : off + 2].copy().view(np.float16).astype(np.float32)  # [nb, 1]


def dq_q4_0(raw):
    b = _blocks(raw, GGMLType.Q4_0)
    d = _f16(b, 0)
    qs = b[:, 2:18]
    lo = (qs & 0xF).astype(np.int32) - 8
    hi = (qs >> 4).astype(np.int32) - 8
    return (np.concatenate([lo, hi], 1) * d).astype(np.float32)


def dq_q4_1(raw):
    b = _blocks(raw, GGMLType.Q4_1)
    d, m = _f16(b, 0), _f16(b, 2)
    qs = b[:, 4:20]
    q = np.concatenate([qs & 0xF, qs >> 4], 1).astype(np.float32)
    return (q * d + m).astype(np.float32)


def _q5_high(qh_bytes: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    qh = qh_bytes.copy().view("<u4").reshape(-1, 1).astype(np.uint64)
    j = np.arange(16, dtype=np.uint64)
    h0 = ((qh >> j) << np.uint64(4)) & np.uint64(0x10)
    h1 = (qh >> (j + np.uint64(12))) & np.uint64(0x10)
    return h0.astype(np.int32), h1.astype(np.int32)


def dq_q5_0(raw):
    b = _blocks(raw, GGMLType.Q5_0)
    d = _f16(b, 0)
    h0, h1 = _q5_high(b[:, 2:6])
    qs = b[:, 6:22].astype(np.int32)
    x0 = ((qs & 0xF) | h0) - 16
    x1 = ((qs >> 4) | h1) - 16
    return (np.concatenate([x0, x1], 1) * d).astype(np.float32)


def dq_q5_1(raw):
    b = _blocks(raw, GGMLType.Q5_1)
    d, m = _f16(b, 0), _f16(b, 2)
    h0, h1 = _q5_high(b[:, 4:8])
    qs = b[:, 8:24].astype(np.int32)
    x0 = (qs & 0xF) | h0
    x1 = (qs >> 4) | h1
    return (np.concatenate([x0, x1], 1) * d + m).astype(np.float32)


def dq_q8_0(raw):
    b = _blocks(raw, GGMLType.Q8_0)
    d = _f16(b, 0)
    return (b[:, 2:34].view(np.int8).astype(np.float32) * d).astype(np.float32)


def dq_q8_1(raw):
    b = _blocks(raw, GGMLType.Q8_1)
    d = _f16(b, 0)
    return (b[:, 4:36].view(np.int8).astype(np.float32) * d).astype(np.float32)


def scale_min_k4(scales: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Unpack the 12-byte K-quant scale field into 8 (scale, min) 6-bit pairs."""
    q = scales.astype(np.int32)
    sc = np.empty((q.shape[0], 8), np.int32)
    mn = np.empty((q.shape[0], 8), np.int32)
    for j in range(8):
        if j < 4:
            sc[:, j] = q[:, j] & 63
            mn[:, j] = q[:, j + 4] & 63
        else:
            sc[:, j] = (q[:, j + 4] & 0xF) | ((q[:, j - 4] >> 6) << 4)
            mn[:, j] = (q[:, j + 4] >> 4) | ((q[:, j] >> 6) << 4)
    return sc, mn


def dq_q4_k(raw):
    b = _blocks(raw, GGMLType.Q4_K)
    d, dmin = _f16(b, 0), _f16(b, 2)
    sc, mn = scale_min_k4(b[:, 4:16])
    qs = b[:, 16:144]
    out = np.empty((b.shape[0], QK_K), np.float32)
    for j in range(4):
        q = qs[:, 32 * j : 32 * j + 32]
        d1 = d * sc[:, 2 * j : 2 * j + 1]
        m1 = dmin * mn[:, 2 * j : 2 * j + 1]
        d2 = d * sc[:, 2 * j + 1 : 2 * j + 2]
        m2 = dmin * mn[:, 2 * j + 1 : 2 * j + 2]
        out[:, 64 * j : 64 * j + 32] = d1 * (q & 0xF) - m1
        out[:, 64 * j + 32 : 64 * j + 64] = d2 * (q >> 4) - m2
    return out


def dq_q5_k(raw):
    b = _blocks(raw, GGMLType.Q5_K)
    d, dmin = _f16(b, 0), _f16(b, 2)
    sc, mn = scale_min_k4(b[:, 4:16])
    qh = b[:, 16:48]
    ql = b[:, 48:176]
    out = np.empty((b.shape[0], QK_K), np.float32)
    for j in range(4):
        q = ql[:, 32 * j : 32 * j + 32].astype(np.int32)
        u1, u2 = 1 << (2 * j), 2 << (2 * j)
        h1 = np.where(qh & u1, 16, 0)
        h2 = np.where(qh & u2, 16, 0)
        out[:, 64 * j : 64 * j + 32] = d * sc[:, 2 * j : 2 * j + 1] * ((q & 0xF) + h1) - dmin * mn[:, 2 * j : 2 * j + 1]
        out[:, 64 * j + 32 : 64 * j + 64] = d * sc[:, 2 * j + 1 : 2 * j + 2] * ((q >> 4) + h2) - dmin * mn[:, 2 * j + 1 : 2 * j + 2]
    return out


def dq_q6_k(raw):
    b = _blocks(raw, GGMLType.Q6_K)
    ql_all = b[:, 0:128].astype(np.int32)
    qh_all = b[:, 128:192].astype(np.int32)
    sc_all = b[:, 192:208].view(np.int8).astype(np.float32)
    d = _f16(b, 208)
    out = np.empty((b.shape[0], QK_K), np.float32)
    for n in range(2):
        ql = ql_all[:, 64 * n : 64 * n + 64]
        qh = qh_all[:, 32 * n : 32 * n + 32]
        sc = sc_all[:, 8 * n : 8 * n + 8]
        l = np.arange(32)
        isx = l // 16
        q1 = ((ql[:, 0:32] & 0xF) | (((qh >> 0) & 3) << 4)) - 32
        q2 = ((ql[:, 32:64] & 0xF) | (((qh >> 2) & 3) << 4)) - 32
        q3 = ((ql[:, 0:32] >> 4) | (((qh >> 4) & 3) << 4)) - 32
        q4 = ((ql[:, 32:64] >> 4) | (((qh >> 6) & 3) << 4)) - 32
        base = 128 * n
        out[:, base + 0 : base + 32] = d * sc[:, isx + 0] * q1
        out[:, base + 32 : base + 64] = d * sc[:, isx + 2] * q2
        out[:, base + 64 : base + 96] = d * sc[:, isx + 4] * q3
        out[:, base + 96 : base + 128] = d * sc[:, isx + 6] * q4
    return out


def dq_q2_k(raw):
    b = _blocks(raw, GGMLType.Q2_K)
    scales = b[:, 0:16].astype(np.int32)
    qs = b[:, 16:80].astype(np.int32)
    d, dmin = _f16(b, 80), _f16(b, 82)
    out = np.empty((b.shape[0], QK_K), np.float32)
    y = 0
    isx = 0
    for n in range(2):
        q = qs[:, 32 * n : 32 * n + 32]
        for j in range(4):
            shift = 2 * j
            for half in range(2):
                sc = scales[:, isx : isx + 1]
                isx += 1
                dl = d * (sc & 0xF)
                ml = dmin * (sc >> 4)
                out[:, y : y + 16] = dl * ((q[:, 16 * half : 16 * half + 16] >> shift) & 3) - ml
                y += 16
    return out


def q3_k_scales(sc12: np.ndarray) -> np.ndarray:
    a = sc12.copy().view("<u4").reshape(-1, 3).astype(np.uint32)
    k1, k2 = np.uint32(0x03030303), np.uint32(0x0F0F0F0F)
    tmp = a[:, 2]
    aux = np.empty((a.shape[0], 4), np.uint32)
    aux[:, 2] = ((a[:, 0] >> 4) & k2) | (((tmp >> 4) & k1) << 4)
    aux[:, 3] = ((a[:, 1] >> 4) & k2) | (((tmp >> 6) & k1) << 4)
    aux[:, 0] = (a[:, 0] & k2) | (((tmp >> 0) & k1) << 4)
    aux[:, 1] = (a[:, 1] & k2) | (((tmp >> 2) & k1) << 4)
    return aux.view(np.int8).reshape(-1, 16).astype(np.int32) - 32


def dq_q3_k(raw):
    b = _blocks(raw, GGMLType.Q3_K)
    hm = b[:, 0:32].astype(np.int32)
    qs = b[:, 32:96].astype(np.int32)
    scales = q3_k_scales(b[:, 96:108])
    d = _f16(b, 108)
    out = np.empty((b.shape[0], QK_K), np.float32)
    y = 0
    isx = 0
    m = 1
    for n in range(2):
        q = qs[:, 32 * n : 32 * n + 32]
        for j in range(4):
            shift = 2 * j
            for half in range(2):
                sl = slice(16 * half, 16 * half + 16)
                dl = d * scales[:, isx : isx + 1]
                isx += 1
                out[:, y : y + 16] = dl * (((q[:, sl] >> shift) & 3) - np.where(hm[:, sl] & m, 0, 4))
                y += 16
            m <<= 1
    return out


def dq_q8_k(raw):
    b = _blocks(raw, GGMLType.Q8_K)
    d = b[:, 0:4].copy().view("<f4").astype(np.float32)
    return (b[:, 4:260].view(np.int8).astype(np.float32) * d).astype(np.float32)


_KV = np.array(KVALUES_IQ4NL, np.float32)


def dq_iq4_nl(raw):
    b = _blocks(raw, GGMLType.IQ4_NL)
    d = _f16(b, 0)
    qs = b[:, 2:18]
    return (np.concatenate([_KV[qs & 0xF], _KV[qs >> 4]], 1) * d).astype(np.float32)


def dq_iq4_xs(raw):
    b = _blocks(raw, GGMLType.IQ4_XS)
    d = _f16(b, 0)
    sh = b[:, 2:4].copy().view("<u2").astype(np.int32)  # [nb,1]
    sl = b[:, 4:8].astype(np.int32)
    qs = b[:, 8:136]
    out = np.empty((b.shape[0], QK_K), np.float32)
    for ib in range(8):
        ls = ((sl[:, ib // 2] >> (4 * (ib % 2))) & 0xF) | (((sh[:, 0] >> (2 * ib)) & 3) << 4)
        dl = d[:, 0] * (ls - 32)
        q = qs[:, 16 * ib : 16 * ib + 16]
        out[:, 32 * ib : 32 * ib + 16] = dl[:, None] * _KV[q & 0xF]
        out[:, 32 * ib + 16 : 32 * ib + 32] = dl[:, None] * _KV[q >> 4]
    return out


_DQ = {
    GGMLType.Q4_0: dq_q4_0,
    GGMLType.Q4_1: dq_q4_1,
    GGMLType.Q5_0: dq_q5_0,
    GGMLType.Q5_1: dq_q5_1,
    GGMLType.Q8_0: dq_q8_0,
    GGMLType.Q8_1: dq_q8_1,
    GGMLType.Q2_K: dq_q2_k,
    GGMLType.Q3_K: dq_q3_k,
    GGMLType.Q4_K: dq_q4_k,
    GGMLType.Q5_K: dq_q5_k,
    GGMLType.Q6_K: dq_q6_k,
    GGMLType.Q8_K: dq_q8_k,
    GGMLType.IQ4_NL: dq_iq4_nl,
    GGMLType.IQ4_XS: dq_iq4_xs,
}


def _tq(name):
    def f(raw):
        from . import ternary

        return getattr(ternary, name)(raw)
    return f


_DQ[GGMLType.TQ1_0] = _tq("dq_tq1_0")
_DQ[GGMLType.TQ2_0] = _tq("dq_tq2_0")


def dequantize(raw: np.ndarray, t: GGMLType, shape: tuple[int, ...] | None = None) -> np.ndarray:
    """Packed GGUF bytes of type ``t`` -> float32 (reshaped to row-major ``shape`` if given)."""
    t = GGMLType(t)
    r = np.ascontiguousarray(raw)
    if t == GGMLType.F32:
        out = r.view(np.uint8).view("<f4").astype(np.float32)
    elif t == GGMLType.F16:
        out = r.view(np.uint8).view("<f2").astype(np.float32)
    elif t == GGMLType.BF16:
        u = r.view(np.uint8).view("<u2").astype(np.uint32) << 16
        out = u.view(np.float32)
    elif t == GGMLType.F64:
        out = r.view(np.uint8).view("<f8").astype(np.float32)
    elif t in (GGMLType.I8, GGMLType.I16, GGMLType.I32, GGMLType.I64):
        dt = {GGMLType.I8: "<i1", GGMLType.I16: "<i2", GGMLType.I32: "<i4", GGMLType.I64: "<i8"}[t]
        out = r.view(np.uint8).view(dt).astype(np.float32)
    elif t in _DQ:
        out = _DQ[t](r).reshape(-1)
    elif TYPE_TRAITS.get(t) is not None and TYPE_TRAITS[t].row_meta:
        from .ik_quants import DQ_IK

        if shape is None:
            raise ValueError(f"dequantize: {t.name} has a per-row scale, pass the shape")
        out = DQ_IK[t](r, int(shape[-1])).reshape(-1)
    else:
        raise NotImplementedError(f"dequantize: {t.name}")
    return out.reshape(shape) if shape is not None else out


def supported_dequant_types() -> list[GGMLType]:
    return [GGMLType.F32, GGMLType.F16, GGMLType.BF16, *list(_DQ), GGMLType.IQ4_KS, GGMLType.IQ3_KS,
            GGMLType.IQ2_KS]
