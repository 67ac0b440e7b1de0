"""Ternary GGUF types TQ1_0 / TQ2_0 (weights in {-1, 0, +1} x one fp16 scale per 256 values).

Parity: the reference lists ``TQ1_0`` / ``TQ2_0`` as quantization tags only
(``barq_core/src/quant.rs:46-47,78-79,111-112``).  Here files holding them are read bit-exactly and
written, following the published ggml block layouts (ggml type ids 34 and 35):

* TQ2_0 (66 bytes / 256 values): ``qs[64]`` then fp16 ``d``.  Byte ``j + m`` of the 32-byte group
  ``j`` holds, in its bit pairs ``l = 0..3``, the codes of values ``4j + 32l + m``; value =
  (code - 1) * d.
* TQ1_0 (54 bytes / 256 values): ``qs[48]``, ``qh[4]``, fp16 ``d``.  Five ternary digits per byte
  (four in ``qh``), stored as a base-3 fraction: a byte ``b`` encodes digits t0..t4 as
  ceil((t0*81 + t1*27 + t2*9 + t3*3 + t4) * 256 / 243), so digit n is recovered as
  ``((b * 3^n) mod 256) * 3 >> 8``.  Bytes 0..31 carry values n*32 + m (n = digit), bytes 32..47
  values 160 + n*16 + m, and ``qh[j]`` values 240 + n*4 + j for n = 0..3.

Both import losslessly into Q4_0 for the device kernels: a ternary value (t-1)*d is a Q4_0 code
t+7 with the same fp16 scale in each of the eight 32-value blocks.
"""
from __future__ import annotations

import numpy as np

QK = 256
TQ1_BYTES, TQ2_BYTES = 48 + 4 + 2, 64 + 2
_POW3 = np.array([1, 3, 9, 27, 81, 243], dtype=np.uint16)


def _f16(b: np.ndarray, off: int) -> np.ndarray:
    return b[:, off:off + 2].copy().view(np.float16).astype(np.float32)  # [nb, 1]


def _digits(bytes_: np.ndarray, n_digits: int) -> np.ndarray:
    """[..., k] bytes -> [..., n_digits, k] ternary digits (0, 1, 2), most significant first."""
    q = (bytes_.astype(np.uint16)[..., None, :] * _POW3[:n_digits, None]) & 0xFF
    return ((q * 3) >> 8).astype(np.int8)


def dq_tq2_0(raw: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(raw).view(np.uint8).reshape(-1, TQ2_BYTES)
    d = _f16(b, 64)
    qs = b[:, :64].reshape(-1, 2, 32)  # [nb, group j, m]
    codes = (qs[:, :, None, :] >> (2 * np.arange(4, dtype=np.uint8))[None, None, :, None]) & 3  # [nb, j, l, m]
    return ((codes.reshape(-1, QK).astype(np.float32) - 1.0) * d).astype(np.float32)


def dq_tq1_0(raw: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(raw).view(np.uint8).reshape(-1, TQ1_BYTES)
    d = _f16(b, 52)
    a = _digits(b[:, 0:32], 5).reshape(-1, 160)   # value n*32 + m
    c = _digits(b[:, 32:48], 5).reshape(-1, 80)   # value 160 + n*16 + m
    h = _digits(b[:, 48:52], 4).reshape(-1, 16)   # value 240 + n*4 + j
    codes = np.concatenate([a, c, h], 1).astype(np.float32)
    return ((codes - 1.0) * d).astype(np.float32)


def _scale_codes(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    x = np.asarray(x, np.float32).reshape(-1, QK)
    amax = np.abs(x).max(1, keepdims=True)
    d16 = amax.astype(np.float16)
    inv = np.where(amax > 0, 1.0 / np.maximum(amax, 1e-30), 0.0)
    codes = (np.clip(np.rint(x * inv), -1, 1) + 1).astype(np.uint16)  # 0, 1, 2
    return codes, d16


def q_tq2_0(x: np.ndarray) -> np.ndarray:
    codes, d16 = _scale_codes(x)
    c = codes.reshape(-1, 2, 4, 32)  # [nb, j, l, m]
    qs = (c << (2 * np.arange(4, dtype=np.uint16))[None, None, :, None]).sum(2).astype(np.uint8)  # [nb, j, m]
    return np.concatenate([qs.reshape(-1, 64), d16.view(np.uint8).reshape(-1, 2)], 1).reshape(-1)


def _pack_base3(codes: np.ndarray, n_digits: int) -> np.ndarray:
    """[..., n_digits, k] digits -> [..., k] bytes (digit 0 most significant, padded to 5 digits)."""
    v = np.zeros(codes.shape[:-2] + codes.shape[-1:], dtype=np.uint32)
    for n in range(n_digits):
        v = v * 3 + codes[..., n, :]
    v = v * (3 ** (5 - n_digits))
    return ((v * 256 + 242) // 243).astype(np.uint8)


def q_tq1_0(x: np.ndarray) -> np.ndarray:
    codes, d16 = _scale_codes(x)
    a = _pack_base3(codes[:, :160].reshape(-1, 5, 32), 5)
    c = _pack_base3(codes[:, 160:240].reshape(-1, 5, 16), 5)
    h = _pack_base3(codes[:, 240:].reshape(-1, 4, 4), 4)
    return np.concatenate([a, c, h, d16.view(np.uint8).reshape(-1, 2)], 1).reshape(-1)


def to_q4_0(raw: np.ndarray, tq1: bool) -> np.ndarray:
    """Lossless TQ -> Q4_0 repack: the same values, eight 32-value Q4_0 blocks per TQ block."""
    b = np.ascontiguousarray(raw).view(np.uint8).reshape(-1, TQ1_BYTES if tq1 else TQ2_BYTES)
    d16 = b[:, -2:].copy()  # fp16 scale bytes
    vals = dq_tq1_0(b) if tq1 else dq_tq2_0(b)
    d = d16.view(np.float16).astype(np.float32)
    codes = np.where(d > 0, np.rint(vals / np.where(d > 0, d, 1.0)), 0).astype(np.int16) + 8  # 7, 8, 9
    codes = codes.reshape(-1, 8, 32).astype(np.uint8)
    qs = (codes[:, :, :16] | (codes[:, :, 16:] << 4)).astype(np.uint8)  # low nibble j, high nibble j+16
    dd = np.repeat(d16[:, None, :], 8, axis=1)
    return np.concatenate([dd, qs], 2).reshape(-1)
