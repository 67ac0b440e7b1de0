"""Numpy model of the Blackwell data movement and tensor-core instructions the tcgen05 kernels use,
for CPU tests of their shared-memory layouts, UMMA descriptors and TMEM column plans.

Modelled (from the PTX ISA and CUTLASS's canonical UMMA layouts, cute/atom/mma_traits_sm100.hpp):

* shared memory: a byte-addressed array of 16-bit operands; the 128-byte swizzle maps byte address
  ``a`` to ``a ^ (((a >> 7) & 7) << 4)`` (16-byte chunk index XOR the 128-byte row index mod 8);
* ``cp.async.bulk.tensor.2d`` with SWIZZLE_128B: box element (row, col) of a 64-column 16-bit box
  lands at ``swz(dst + 128 row + 2 col)`` (dst 1024-byte aligned);
* UMMA shared-memory descriptors (start >> 4 in bits 0-13, LBO >> 4 in 16-29, SBO >> 4 in 32-45,
  layout in 61-63, 2 = SWIZZLE_128B): a K-major operand element (row, k) sits at
  ``swz(start + (row / 8) SBO + 128 (row % 8) + 2 k)``; an MN-major one (mn, k) at
  ``swz(start + (mn / 64) LBO + (k / 8) SBO + 128 (k % 8) + 2 (mn % 64))``;
* the kind::f16 instruction descriptor (D format bits 4-5, A / B format bits 7-9 / 10-12 with
  0 = f16 and 1 = bf16, A / B major bits 15 / 16, N >> 3 in bits 17-22, M >> 4 in bits 24-28);
* TMEM as 128 lanes x 512 columns of 32 bits, addresses ``(lane << 16) | column``; an accumulator
  D[m][n] is lane m, column d + n (f32); a TMEM A operand A[m][k] is the low (k even) or high half
  of lane m, column a + k / 2.

The model is first checked on the addressing of the tcgen05 GEMM (``csrc/kernels/gemm_tc.cu``),
whose results are verified on B200s (``tests/test_tcgen05_emulation_cpu.py``).
"""
from __future__ import annotations

import numpy as np

SMEM_BYTES = 256 * 1024


def swz(addr):
    addr = np.asarray(addr, dtype=np.int64)
    return addr ^ (((addr >> 7) & 7) << 4)


def to_bits(x, dtype: str) -> np.ndarray:
    """Round floats to fp16 / bf16 (nearest even) and return their 16-bit patterns."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp16":
        return x.astype(np.float16).view(np.uint16)
    u = x.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def from_bits(b, dtype: str) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    if dtype == "fp16":
        return b.view(np.float16).astype(np.float64)
    return (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


class Smem:
    def __init__(self):
        self.h = np.zeros(SMEM_BYTES // 2, dtype=np.uint16)

    def store16(self, byte_addr, bits):
        self.h[np.asarray(byte_addr) // 2] = bits

    def load16(self, byte_addr):
        return self.h[np.asarray(byte_addr) // 2]

    def tma_2d_sw128(self, dst: int, box_bits: np.ndarray) -> None:
        """A [rows, 64] box of 16-bit values written as cp.async.bulk.tensor with SWIZZLE_128B."""
        assert dst % 1024 == 0 and box_bits.shape[1] == 64
        rows = box_bits.shape[0]
        r, c = np.meshgrid(np.arange(rows), np.arange(64), indexing="ij")
        self.store16(swz(dst + 128 * r + 2 * c), box_bits)


def desc_fields(desc: int):
    start = (desc & 0x3FFF) << 4
    lbo = ((desc >> 16) & 0x3FFF) << 4
    sbo = ((desc >> 32) & 0x3FFF) << 4
    layout = (desc >> 61) & 7
    version = (desc >> 46) & 3
    return start, lbo, sbo, layout, version


def idesc_fields(idesc: int):
    return dict(d_f32=((idesc >> 4) & 3) == 1, a_fmt=(idesc >> 7) & 7, b_fmt=(idesc >> 10) & 7,
                a_mn=(idesc >> 15) & 1, b_mn=(idesc >> 16) & 1, N=((idesc >> 17) & 0x3F) << 3,
                M=((idesc >> 24) & 0x1F) << 4)


def read_operand(smem: Smem, desc: int, rows: int, mn_major: bool, dtype: str) -> np.ndarray:
    """[rows, 16] operand values (K = 16 for kind::f16) named by a SWIZZLE_128B descriptor."""
    start, lbo, sbo, layout, version = desc_fields(desc)
    assert layout == 2 and version == 1, "only SWIZZLE_128B sm_100 descriptors are modelled"
    m, k = np.meshgrid(np.arange(rows), np.arange(16), indexing="ij")
    if mn_major:
        addr = start + (m // 64) * lbo + (k // 8) * sbo + 128 * (k % 8) + 2 * (m % 64)
    else:
        addr = start + (m // 8) * sbo + 128 * (m % 8) + 2 * k
    return from_bits(smem.load16(swz(addr)), dtype)


class Tmem:
    def __init__(self):
        self.w = np.zeros((128, 512), dtype=np.uint32)

    @staticmethod
    def split(addr: int):
        return addr >> 16, addr & 0xFFFF

    def ld_f32(self, lane0: int, col: int, ncols: int) -> np.ndarray:
        """32 lanes x ncols columns as f32 (tcgen05.ld 32x32b)."""
        return self.w[lane0:lane0 + 32, col:col + ncols].view(np.float32).astype(np.float64)

    def st_u32(self, lane0: int, col: int, words: np.ndarray) -> None:
        self.w[lane0:lane0 + words.shape[0], col:col + words.shape[1]] = words

    def a_operand(self, addr: int, dtype: str) -> np.ndarray:
        """[128, 16] A operand from TMEM (two 16-bit values per column, even k low)."""
        _, col = self.split(addr)
        words = self.w[:, col:col + 8]
        lo = from_bits((words & 0xFFFF).astype(np.uint16), dtype)
        hi = from_bits((words >> 16).astype(np.uint16), dtype)
        out = np.empty((128, 16))
        out[:, 0::2], out[:, 1::2] = lo, hi
        return out


def mma(tmem: Tmem, d_addr: int, a, b_desc: int, idesc: int, accumulate: bool, smem: Smem,
        a_tmem: bool = False) -> None:
    """tcgen05.mma.cta_group::1.kind::f16: D (+)= A B^T with A [M, 16] and B [N, 16]."""
    f = idesc_fields(idesc)
    assert f["d_f32"] and f["M"] == 128 and f["a_fmt"] == f["b_fmt"], "same A / B type, M = 128, f32 D"
    dtype = "bf16" if f["a_fmt"] == 1 else "fp16"
    A = tmem.a_operand(a, dtype) if a_tmem else read_operand(smem, a, 128, bool(f["a_mn"]), dtype)
    B = read_operand(smem, b_desc, f["N"], bool(f["b_mn"]), dtype)
    lane0, col = Tmem.split(d_addr)
    assert lane0 == 0
    acc = tmem.w[:, col:col + f["N"]].view(np.float32).astype(np.float64) if accumulate else 0.0
    tmem.w[:, col:col + f["N"]] = (acc + A @ B.T).astype(np.float32).view(np.uint32)


# Descriptor builders with the kernels' own formulas (csrc/kernels/tc_common.cuh).
def umma_desc_sw128(saddr: int) -> int:
    return ((saddr >> 4) & 0x3FFF) | (1 << 16) | ((1024 >> 4) << 32) | (1 << 46) | (2 << 61)


def umma_desc_sw128_mn(saddr: int, lbo: int) -> int:
    return ((saddr >> 4) & 0x3FFF) | (((lbo >> 4) & 0x3FFF) << 16) | ((1024 >> 4) << 32) | (1 << 46) | (2 << 61)


def idesc_bf16(M: int, N: int) -> int:
    return (1 << 4) | (1 << 7) | (1 << 10) | ((N >> 3) << 17) | ((M >> 4) << 24)


def idesc_f16(M: int, N: int) -> int:
    return (1 << 4) | ((N >> 3) << 17) | ((M >> 4) << 24)


IDESC_B_MAJOR_MN = 1 << 16
