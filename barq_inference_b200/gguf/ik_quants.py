"""ik_llama.cpp row-scaled quant types (IQ4_KS, IQ3_KS, IQ2_KS) and the Q4_K_R4 row repack.

Parity: ``quant/src/iq.rs:120-360`` (dequantizers), ``iq.rs:430-700`` (quantizers) and
``quant/src/ik_quant.rs:187-305`` (``quantize_model_ik`` / ``repack_model_cpu``).

Formats (ik_llama's published block definitions; every row starts with a row scale):

* IQ4_KS, 4.25 bpw: row = f32 ``d`` + blocks of 256 = ``scales[8]`` + ``qs[128]``.  Block ``b``
  (32 values) has scale ``d * ((scales[b] & 254) - 127)`` and codebook half ``scales[b] & 1``;
  value ``j < 16`` is the low nibble of ``qs[16b + j]``, value ``j + 16`` the high nibble.
  (The reference's dequantizer interleaves the nibbles instead, ``iq.rs:165-171``; files written
  by ik_llama use the split order, which is what is read here.)
* IQ2_KS, 2.19 bpw: row = f16 ``d`` + blocks of 256 = ``extra`` (u16) + ``scales[4]`` + ``qs[64]``.
  Block ``b``: 5-bit scale = nibble ``b & 1`` of ``scales[b >> 1]`` | bit ``8 + b`` of ``extra``
  << 4, value scale ``d * (ls - 16)``; codebook half = bit ``b`` of ``extra``; 2-bit index of
  value ``j`` = ``qs[32 (b >> 2) + j] >> 2 (b & 3)``.
* IQ3_KS, 3.19 bpw: row = f16 ``d`` + blocks of 256 = ``extra`` + ``scales[4]`` + ``qs[64]`` +
  ``qh[32]``.  Block ``b``: 5-bit scale = nibble ``b >> 2`` of ``scales[b & 3]`` | bit ``b`` of
  ``extra`` << 4; codebook half = bit ``8 + b`` of ``extra``; 3-bit index of value ``j`` =
  ``qs[32 (b >> 2) + j] >> 2 (b & 3)`` (2 bits) | bit ``b`` of ``qh[j]`` << 2.
* Q4_K_R4 (CPU repack, archive-only): four rows' Q4_K super-blocks of one 256-column slice packed
  together, 576 bytes = ``d[4]`` + ``dmin[4]`` (f16) + the four 12-byte scale fields + the four
  rows' 128 quant bytes interleaved in 16-byte pieces.  Lossless both ways, so a repacked file
  imports back to Q4_K exactly (the device already keeps its own tiled layout).

On the GPU these types are imported by requantizing to a type the kernels stream
(:data:`IK_IMPORT`); the CPU oracle reads them directly.
"""
from __future__ import annotations

import os

import numpy as np
import torch

from .constants import KVALUES_IQ2NL, KVALUES_IQ3NL, KVALUES_IQ4K, QK_K, TYPE_TRAITS, GGMLType, row_nbytes

_V4 = np.array(KVALUES_IQ4K, np.float32)
_V2 = np.array(KVALUES_IQ2NL, np.float32)
_V3 = np.array(KVALUES_IQ3NL, np.float32)

IK_TYPES = (GGMLType.IQ4_KS, GGMLType.IQ3_KS, GGMLType.IQ2_KS)

# device import: ik type -> type the GEMV/GEMM kernels stream (override: BARQ_IK_IMPORT=q8_0|q6_k|q4_k)
IK_IMPORT = {GGMLType.IQ4_KS: GGMLType.Q6_K, GGMLType.IQ3_KS: GGMLType.Q4_K, GGMLType.IQ2_KS: GGMLType.Q4_K}


def import_type(t: GGMLType) -> GGMLType:
    env = os.environ.get("BARQ_IK_IMPORT")
    if env:
        from .constants import QUANT_NAME_TO_TYPE

        return QUANT_NAME_TO_TYPE[env.lower()]
    return IK_IMPORT[GGMLType(t)]


def _split_rows(raw: np.ndarray, t: GGMLType, ne0: int) -> tuple[np.ndarray, np.ndarray]:
    """-> (row scale [R] f32, blocks [R * nb, type_size] u8)."""
    tr = TYPE_TRAITS[t]
    rb = row_nbytes(t, ne0)
    r = np.ascontiguousarray(raw).view(np.uint8).reshape(-1)
    if r.size % rb:
        raise ValueError(f"{t.name}: {r.size} bytes is not a whole number of {rb}-byte rows")
    r = r.reshape(-1, rb)
    meta = r[:, : tr.row_meta].copy()
    d = meta.view("<f4" if tr.row_meta == 4 else "<f2").astype(np.float32).reshape(-1)
    return d, r[:, tr.row_meta:].reshape(-1, tr.type_size)


def dq_iq4_ks(raw: np.ndarray, ne0: int) -> np.ndarray:
    d, b = _split_rows(raw, GGMLType.IQ4_KS, ne0)
    nb = ne0 // QK_K
    dd = np.repeat(d, nb)[:, None]  # [blocks, 1]
    sc = b[:, :8].astype(np.int32)
    qs = b[:, 8:]
    out = np.empty((b.shape[0], QK_K), np.float32)
    for ib in range(8):
        dl = dd[:, 0] * ((sc[:, ib] & 254) - 127)
        off = (sc[:, ib] & 1)[:, None] * 16
        q = qs[:, 16 * ib: 16 * ib + 16].astype(np.int32)
        out[:, 32 * ib: 32 * ib + 16] = dl[:, None] * _V4[off + (q & 0xF)]
        out[:, 32 * ib + 16: 32 * ib + 32] = dl[:, None] * _V4[off + (q >> 4)]
    return out.reshape(-1, ne0)


def _ks_scales(b: np.ndarray, iq3: bool) -> tuple[np.ndarray, np.ndarray]:
    """-> (5-bit scale - 16 [blocks, 8], codebook half [blocks, 8]) of IQ2_KS / IQ3_KS."""
    extra = b[:, 0:2].copy().view("<u2").astype(np.int32)[:, 0]
    sc = b[:, 2:6].astype(np.int32)
    ls = np.empty((b.shape[0], 8), np.int32)
    half = np.empty((b.shape[0], 8), np.int32)
    for blk in range(8):
        if iq3:
            nib = (sc[:, blk & 3] >> (4 * (blk >> 2))) & 0xF
            ls[:, blk] = nib | (((extra >> blk) & 1) << 4)
            half[:, blk] = (extra >> (8 + blk)) & 1
        else:
            nib = (sc[:, blk >> 1] >> (4 * (blk & 1))) & 0xF
            ls[:, blk] = nib | (((extra >> (8 + blk)) & 1) << 4)
            half[:, blk] = (extra >> blk) & 1
    return ls - 16, half


def dq_iq2_ks(raw: np.ndarray, ne0: int) -> np.ndarray:
    d, b = _split_rows(raw, GGMLType.IQ2_KS, ne0)
    dd = np.repeat(d, ne0 // QK_K)
    ls, half = _ks_scales(b, iq3=False)
    qs = b[:, 6:70].astype(np.int32)
    out = np.empty((b.shape[0], QK_K), np.float32)
    for blk in range(8):
        q = (qs[:, 32 * (blk >> 2): 32 * (blk >> 2) + 32] >> (2 * (blk & 3))) & 3
        out[:, 32 * blk: 32 * blk + 32] = (dd * ls[:, blk])[:, None] * _V2[half[:, blk:blk + 1] * 4 + q]
    return out.reshape(-1, ne0)


def dq_iq3_ks(raw: np.ndarray, ne0: int) -> np.ndarray:
    d, b = _split_rows(raw, GGMLType.IQ3_KS, ne0)
    dd = np.repeat(d, ne0 // QK_K)
    ls, half = _ks_scales(b, iq3=True)
    qs = b[:, 6:70].astype(np.int32)
    qh = b[:, 70:102].astype(np.int32)
    out = np.empty((b.shape[0], QK_K), np.float32)
    for blk in range(8):
        q = ((qs[:, 32 * (blk >> 2): 32 * (blk >> 2) + 32] >> (2 * (blk & 3))) & 3) | (((qh >> blk) & 1) << 2)
        out[:, 32 * blk: 32 * blk + 32] = (dd * ls[:, blk])[:, None] * _V3[half[:, blk:blk + 1] * 8 + q]
    return out.reshape(-1, ne0)


DQ_IK = {GGMLType.IQ4_KS: dq_iq4_ks, GGMLType.IQ2_KS: dq_iq2_ks, GGMLType.IQ3_KS: dq_iq3_ks}


# ---------------------------------------------------------------------------------- quantizers
def _nearest(x: torch.Tensor, cb: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """x [..., n] (already divided by the block scale) -> (index into cb, squared error) per value."""
    dist = (x[..., None] - cb) ** 2
    err, idx = dist.min(-1)
    return idx, err


def _block_search(b: torch.Tensor, s: torch.Tensor, cb: torch.Tensor, n_half: int):
    """Pick per block the codebook half with the lower error at block scale ``s``.
    b [nb, 32], s [nb] -> (indices [nb, 32] within the half, half [nb])."""
    safe = torch.where(s == 0, torch.ones_like(s), s)[:, None]
    x = b / safe
    i0, e0 = _nearest(x, cb[:n_half])
    i1, e1 = _nearest(x, cb[n_half:])
    use1 = (e1 * safe ** 2).sum(-1) < (e0 * safe ** 2).sum(-1)
    return torch.where(use1[:, None], i1, i0), use1.long()


_SEARCH = (0.75, 0.8, 0.85, 0.9, 0.95, 1.0, 1.05)


def _search_levels(b: torch.Tensor, s_blk: torch.Tensor, dd: torch.Tensor, cb: torch.Tensor, n_half: int,
                   to_level):
    """Try the block scale ``s_blk`` times each factor of _SEARCH (the extreme value need not land
    on the extreme code); keep per block the (level, indices, half) with the lowest squared error."""
    best = None
    for f in _SEARCH:
        lvl = to_level(s_blk * f, dd)
        s = dd * lvl
        idx, half = _block_search(b, s, cb, n_half)
        vals = cb[half[:, None] * n_half + idx] * s[:, None]
        err = ((vals - b) ** 2).sum(-1)
        if best is None:
            best = [err, lvl, idx, half]
        else:
            m = err < best[0]
            best = [torch.where(m, err, best[0]), torch.where(m, lvl, best[1]),
                    torch.where(m[:, None], idx, best[2]), torch.where(m, half, best[3])]
    return best[1], best[2], best[3]


def _signed_absmax(b: torch.Tensor) -> torch.Tensor:
    return torch.gather(b, -1, b.abs().argmax(-1, keepdim=True))[:, 0]


def _rowwise(x: torch.Tensor) -> tuple[torch.Tensor, int]:
    if x.shape[-1] % QK_K:
        raise ValueError(f"ik quant: last dim {x.shape[-1]} not a multiple of {QK_K}")
    return x.reshape(-1, x.shape[-1]).to(torch.float32), x.shape[-1]


def quantize_iq4_ks(x: torch.Tensor) -> torch.Tensor:
    rows, ne0 = _rowwise(x)
    R = rows.shape[0]
    cb = torch.tensor(KVALUES_IQ4K, dtype=torch.float32, device=rows.device)
    b = rows.reshape(-1, 32)
    s_blk = _signed_absmax(b) / -127.0  # block scale so that the extreme value maps onto -127
    d = s_blk.reshape(R, -1).abs().amax(-1) / 127.0  # row scale: |level| <= 127
    dd = d.repeat_interleave(ne0 // 32)

    def to_level(sb, dd):
        lvl = torch.where(dd > 0, sb / torch.where(dd > 0, dd, torch.ones_like(dd)), torch.zeros_like(dd))
        return (torch.round((lvl + 127) / 2) * 2 - 127).clamp(-127, 127)  # odd levels: (byte & 254) - 127

    lvl, idx, half = _search_levels(b, s_blk, dd, cb, 16, to_level)
    sbyte = ((lvl + 127).to(torch.int32) | half.to(torch.int32)).to(torch.uint8)  # [nb32]
    q = idx.to(torch.uint8)
    qs = (q[:, :16] | (q[:, 16:] << 4)).reshape(-1, 8, 16)
    blocks = torch.cat([sbyte.reshape(-1, 8), qs.reshape(-1, 128)], 1).reshape(R, -1)
    meta = d.reshape(R, 1).contiguous().view(torch.uint8)
    return torch.cat([meta, blocks], 1).reshape(*x.shape[:-1], -1)


def _quantize_ks(x: torch.Tensor, t: GGMLType) -> torch.Tensor:
    iq3 = t == GGMLType.IQ3_KS
    rows, ne0 = _rowwise(x)
    R = rows.shape[0]
    cb = torch.tensor(KVALUES_IQ3NL if iq3 else KVALUES_IQ2NL, dtype=torch.float32, device=rows.device)
    n_half = 8 if iq3 else 4
    b = rows.reshape(-1, 32)
    s_blk = _signed_absmax(b) / cb[0]  # extreme value -> the most negative code
    d = (s_blk.reshape(R, -1).abs().amax(-1) / 16.0).to(torch.float16).to(torch.float32)
    dd = d.repeat_interleave(ne0 // 32)

    def to_level(sb, dd):
        return torch.where(dd > 0, torch.round(sb / torch.where(dd > 0, dd, torch.ones_like(dd))),
                           torch.zeros_like(dd)).clamp(-16, 15)

    lvl, idx, half = _search_levels(b, s_blk, dd, cb, n_half, to_level)
    ls = (lvl + 16).to(torch.int32).reshape(-1, 8)  # [nbk, 8] 5-bit
    half = half.to(torch.int32).reshape(-1, 8)
    q = idx.to(torch.int32).reshape(-1, 8, 32)
    nbk = ls.shape[0]
    extra = torch.zeros(nbk, dtype=torch.int32, device=rows.device)
    scales = torch.zeros(nbk, 4, dtype=torch.int32, device=rows.device)
    qs = torch.zeros(nbk, 2, 32, dtype=torch.int32, device=rows.device)
    qh = torch.zeros(nbk, 32, dtype=torch.int32, device=rows.device)
    for blk in range(8):
        lo, hi = ls[:, blk] & 0xF, ls[:, blk] >> 4
        if iq3:
            scales[:, blk & 3] |= lo << (4 * (blk >> 2))
            extra |= (hi << blk) | (half[:, blk] << (8 + blk))
            qh |= ((q[:, blk] >> 2) & 1) << blk
        else:
            scales[:, blk >> 1] |= lo << (4 * (blk & 1))
            extra |= (hi << (8 + blk)) | (half[:, blk] << blk)
        qs[:, blk >> 2] |= (q[:, blk] & 3) << (2 * (blk & 3))
    ex = torch.stack([extra & 0xFF, extra >> 8], 1)
    parts = [ex, scales, qs.reshape(nbk, 64)] + ([qh] if iq3 else [])
    blocks = torch.cat(parts, 1).to(torch.uint8).reshape(R, -1)
    meta = d.to(torch.float16).reshape(R, 1).contiguous().view(torch.uint8)
    return torch.cat([meta, blocks], 1).reshape(*x.shape[:-1], -1)


def quantize_iq2_ks(x: torch.Tensor) -> torch.Tensor:
    return _quantize_ks(x, GGMLType.IQ2_KS)


def quantize_iq3_ks(x: torch.Tensor) -> torch.Tensor:
    return _quantize_ks(x, GGMLType.IQ3_KS)


Q_IK = {GGMLType.IQ4_KS: quantize_iq4_ks, GGMLType.IQ2_KS: quantize_iq2_ks, GGMLType.IQ3_KS: quantize_iq3_ks}


# ---------------------------------------------------------------------------------- Q4_K_R4
R4_BYTES = 576  # per group of 4 rows x 256 columns


def repack_q4_k_r4(rows: np.ndarray) -> np.ndarray:
    """Q4_K rows [N, K/256*144] (N % 4 == 0) -> Q4_K_R4 bytes [N/4, K/256*576]."""
    r = np.ascontiguousarray(rows).view(np.uint8)
    N = r.shape[0]
    if N % 4:
        raise ValueError("Q4_K_R4: the row count must be a multiple of 4")
    b = r.reshape(N // 4, 4, -1, 144).transpose(0, 2, 1, 3)  # [g, sb, 4 rows, 144]
    d = b[..., 0:2].reshape(*b.shape[:2], 8)
    dmin = b[..., 2:4].reshape(*b.shape[:2], 8)
    sc = b[..., 4:16].reshape(*b.shape[:2], 48)
    qs = b[..., 16:144].reshape(*b.shape[:2], 4, 8, 16).transpose(0, 1, 3, 2, 4).reshape(*b.shape[:2], 512)
    return np.concatenate([d, dmin, sc, qs], -1).reshape(N // 4, -1)


def unpack_q4_k_r4(packed: np.ndarray, N: int) -> np.ndarray:
    """Inverse of :func:`repack_q4_k_r4` -> Q4_K rows [N, K/256*144]."""
    p = np.ascontiguousarray(packed).view(np.uint8).reshape(N // 4, -1, R4_BYTES)
    G, SB = p.shape[:2]
    d = p[..., 0:8].reshape(G, SB, 4, 2)
    dmin = p[..., 8:16].reshape(G, SB, 4, 2)
    sc = p[..., 16:64].reshape(G, SB, 4, 12)
    qs = p[..., 64:576].reshape(G, SB, 8, 4, 16).transpose(0, 1, 3, 2, 4).reshape(G, SB, 4, 128)
    blk = np.concatenate([d, dmin, sc, qs], -1)  # [G, SB, 4, 144]
    return blk.transpose(0, 2, 1, 3).reshape(N, SB * 144)
