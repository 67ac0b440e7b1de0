"""Lane-level numpy model of the warp-wide tensor-core instructions the attention kernels use, for
CPU tests of their fragment addressing and data flow.

Semantics follow the PTX ISA descriptions of:

* ``ldmatrix.sync.aligned.m8n8.x4.shared.b16`` (optionally ``.trans``): lanes 8 i .. 8 i + 7 give
  the row addresses of matrix i (8 consecutive 16-bit elements each); lane L receives in register
  i the elements (L / 4, 2 (L % 4)) and (L / 4, 2 (L % 4) + 1) of matrix i, or of its transpose
  with ``.trans``;
* ``mma.sync.aligned.m16n8k16.row.col.f32.{f16,bf16}``: with g = L / 4 and t = L % 4, the A
  registers hold A[g][2t..2t+1], A[g+8][2t..], A[g][2t+8..], A[g+8][2t+8..]; the B registers hold
  B[2t..2t+1][g] and B[2t+8..2t+9][g]; the accumulators hold C[g][2t..2t+1] and C[g+8][2t..2t+1].

Registers are modelled as float pairs ``[32, n, 2]`` (lane, register, element); shared memory as a
flat float array of 16-bit operand values (already rounded to the operand type).
"""
from __future__ import annotations

import numpy as np

LANE = np.arange(32)
G, T = LANE // 4, LANE % 4


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float values to fp16 or bf16 (round to nearest even) and back to float64."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "fp16":
        return x.astype(np.float16).astype(np.float64)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32).astype(np.float64)


def ldsm_x4(smem: np.ndarray, addr: np.ndarray, trans: bool = False) -> np.ndarray:
    """addr: [32] element offsets (one row start per lane).  Returns registers [32, 4, 2]."""
    addr = np.asarray(addr)
    rows = smem[addr[:, None] + np.arange(8)[None, :]]  # [32 lanes' rows, 8]
    mats = rows.reshape(4, 8, 8)                        # matrix i = rows of lanes 8i..8i+7
    out = np.empty((32, 4, 2))
    for i in range(4):
        M = mats[i].T if trans else mats[i]
        out[:, i, 0] = M[G, 2 * T]
        out[:, i, 1] = M[G, 2 * T + 1]
    return out


def mma(c: np.ndarray, a: np.ndarray, b: np.ndarray) -> None:
    """c [32, 4] += A (16x16 from a [32, 4, 2]) @ B (16x8 from b [32, 2, 2]), in place."""
    A = np.zeros((16, 16))
    B = np.zeros((16, 8))
    for e in range(2):
        A[G, 2 * T + e] = a[:, 0, e]
        A[G + 8, 2 * T + e] = a[:, 1, e]
        A[G, 2 * T + 8 + e] = a[:, 2, e]
        A[G + 8, 2 * T + 8 + e] = a[:, 3, e]
        B[2 * T + e, G] = b[:, 0, e]
        B[2 * T + 8 + e, G] = b[:, 1, e]
    D = A @ B
    for e in range(2):
        c[:, e] += D[G, 2 * T + e]
        c[:, 2 + e] += D[G + 8, 2 * T + e]


def pack(x: np.ndarray, y: np.ndarray, dtype: str) -> np.ndarray:
    """Two floats per lane rounded to the operand type, as one register [32, 2]."""
    return np.stack([round_to(x, dtype), round_to(y, dtype)], axis=-1)


def shfl_xor_max(v: np.ndarray, masks=(1, 2)) -> np.ndarray:
    for m in masks:
        v = np.maximum(v, v[LANE ^ m])
    return v


def shfl_xor_sum(v: np.ndarray, masks=(1, 2)) -> np.ndarray:
    for m in masks:
        v = v + v[LANE ^ m]
    return v
