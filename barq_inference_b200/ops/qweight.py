"""Quantized weights: GGUF blocks -> planar planes -> the kernels' tiled layout (``csrc/kernels/qtile.cuh``).

``QWeight.from_packed`` splits GGUF blocks into aligned planes on the device without changing a
bit (the planar form is where rows are fused, interleaved or sharded); ``finalize`` then cuts the
planes into 128-row x 256/64-column chunks with row-swizzled 16-byte pieces, the form every kernel
reads.  ``to_gguf_rows`` re-emits the original blocks from either form (tests check the round trip).  Block
types without a kernel format are converted at load: Q3_K to Q6_K (exact), Q5_0 to Q8_0 (exact),
IQ4_XS to IQ4_NL (fp16 rounding of the block scales only), Q2_K / Q4_1 / Q5_1 to Q8_0 (within one
Q8_0 step); F16 / F32 and anything else become bf16
for the dense GEMV/GEMM.  The reference instead dequantizes *everything* to f32 at load
(``barq_core/src/gguf.rs:306-311``).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from ..gguf import TYPE_TRAITS, GGMLType, dequantize
from ..gguf.ik_quants import IK_TYPES

NATIVE = {GGMLType.Q4_0, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q5_K, GGMLType.Q6_K, GGMLType.IQ4_NL}
W_BF16 = 0
# block-quantized GGUF types that are imported to the device by requantization to Q8_0
_REQUANT = {GGMLType.Q5_0, GGMLType.Q5_1, GGMLType.Q4_1, GGMLType.Q2_K, GGMLType.Q3_K, GGMLType.IQ4_XS}


def requant_q8_0(raw: torch.Tensor, t: GGMLType, N: int, K: int) -> torch.Tensor:
    """GGUF rows of a block type without a kernel format -> Q8_0 rows (uint8 [N, K/32*34]).

    Q5_0 is exact: its block (fp16 d, 5-bit q) maps to Q8_0's block (the same d, q - 16 as int8).
    The others are dequantized (the ggml-spec oracle) and requantized to Q8_0, whose 255 levels
    per 32 values add about 1/254 of each block's largest magnitude (plus the fp16 rounding of its scale) -- against the 4..16 levels
    per (sub-)block of the source types.  Costs 8.5 bits per weight on the device instead of 2.6..6."""
    dev = raw.device
    nb = K // 32
    if t == GGMLType.Q5_0:
        b = raw.reshape(N, nb, 22)
        d = b[..., 0:2]
        qh = b[..., 2:6].to(torch.int64)
        qh = qh[..., 0] | (qh[..., 1] << 8) | (qh[..., 2] << 16) | (qh[..., 3] << 24)
        qs = b[..., 6:22].to(torch.int16)
        j = torch.arange(16, device=dev)
        lo = (qs & 0x0F) | (((qh[..., None] >> j) & 1) << 4).to(torch.int16)
        hi = (qs >> 4) | (((qh[..., None] >> (j + 16)) & 1) << 4).to(torch.int16)
        q = (torch.cat([lo, hi], -1) - 16).to(torch.int8).view(torch.uint8)
        return torch.cat([d, q], -1).reshape(N, nb * 34).contiguous()
    from ..gguf import quantize

    w = torch.from_numpy(dequantize(raw.cpu().numpy(), t, (N, K))).to(dev, torch.float32)
    return quantize(w, GGMLType.Q8_0).reshape(N, nb * 34)


def q3_k_as_q6_k(raw: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """Q3_K rows -> Q6_K rows (uint8 [N, K/256*210]), bit-exact.

    Both types are 256-value super-blocks of sixteen 16-value sub-blocks with one fp16 scale d and
    a signed per-sub-block scale: Q3_K stores value = d * (s - 32) * c with a 6-bit s and a code
    c in [-4, 3]; Q6_K stores value = d * sc * (q - 32) with an int8 sc and a 6-bit q.  So d is
    copied, sc = s - 32 and q = c + 32 (28..35), and the ggml-spec dequantization of the result
    equals the source's value for value, while the device streams 6.6 instead of 8.5 bits per weight
    (the Q8_0 import)."""
    from ..gguf.dequant import q3_k_scales

    dev = raw.device
    b = raw.reshape(-1, 110).cpu().numpy()
    nb = b.shape[0]
    hm = b[:, 0:32].astype(np.int32)
    qs = b[:, 32:96].astype(np.int32)
    codes = np.empty((nb, 256), np.int32)
    y = 0
    for n in range(2):  # element order of the Q3_K block: 2 x 4 shifts x 2 halves of 16
        q = qs[:, 32 * n: 32 * n + 32]
        for j in range(4):
            m = 1 << (4 * n + j)
            for half in range(2):
                sl = slice(16 * half, 16 * half + 16)
                codes[:, y:y + 16] = ((q[:, sl] >> (2 * j)) & 3) - np.where(hm[:, sl] & m, 0, 4)
                y += 16
    q6 = codes + 32
    out = np.empty((nb, 210), np.uint8)
    for n in range(2):  # Q6_K packing: low nibbles in ql, the two high bits of 4 values per qh byte
        e1, e2, e3, e4 = (q6[:, 128 * n + 32 * i: 128 * n + 32 * i + 32] for i in range(4))
        out[:, 64 * n: 64 * n + 32] = (e1 & 0xF) | ((e3 & 0xF) << 4)
        out[:, 64 * n + 32: 64 * n + 64] = (e2 & 0xF) | ((e4 & 0xF) << 4)
        out[:, 128 + 32 * n: 128 + 32 * n + 32] = (e1 >> 4) | ((e2 >> 4) << 2) | ((e3 >> 4) << 4) | ((e4 >> 4) << 6)
    out[:, 192:208] = q3_k_scales(b[:, 96:108]).astype(np.int8).view(np.uint8)
    out[:, 208:210] = b[:, 108:110]
    return torch.from_numpy(out).to(dev).reshape(N, K // 256 * 210)


def iq4_xs_as_iq4_nl(raw: torch.Tensor, N: int, K: int) -> torch.Tensor:
    """IQ4_XS rows -> IQ4_NL rows (uint8 [N, K/32*18]).

    An IQ4_XS super-block (fp16 d, eight 6-bit sub-block scales ls, 4-bit codebook codes) is eight
    32-value IQ4_NL blocks with the same codes and the block scale d * (ls - 32) rounded to fp16:
    the only change is that rounding (relative error <= 2^-11, none when ls - 32 is a power of two
    or the product fits fp16's 11-bit significand).  4.5 bits per weight on the device, against 8.5
    for the Q8_0 import, whose per-block error is ~2^-8 of the block maximum."""
    dev = raw.device
    b = raw.reshape(-1, 136).cpu().numpy()
    nb = b.shape[0]
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)  # [nb, 1]
    sh = b[:, 2:4].copy().view("<u2").astype(np.int32)
    sl = b[:, 4:8].astype(np.int32)
    out = np.empty((nb, 8, 18), np.uint8)
    for ib in range(8):
        ls = ((sl[:, ib // 2] >> (4 * (ib % 2))) & 0xF) | (((sh[:, 0] >> (2 * ib)) & 3) << 4)
        out[:, ib, 0:2] = (d[:, 0] * (ls - 32)).astype(np.float16).view(np.uint8).reshape(nb, 2)
        out[:, ib, 2:18] = b[:, 8 + 16 * ib: 8 + 16 * ib + 16]
    return torch.from_numpy(out).to(dev).reshape(N, K // 32 * 18)


def _blocks(raw: torch.Tensor, N: int, t: GGMLType) -> torch.Tensor:
    ts = TYPE_TRAITS[t].type_size
    return raw.reshape(N, -1, ts)


def _u16(x: torch.Tensor) -> torch.Tensor:
    """[..., 2] uint8 -> [...] int16 bit pattern (fp16 scales)."""
    return x.contiguous().view(torch.int16).squeeze(-1)


@dataclass
class QWeight:
    wtype: int  # GGMLType value for native types, 0 for bf16
    N: int
    K: int
    p0: torch.Tensor
    p1: torch.Tensor | None = None
    p2: torch.Tensor | None = None
    d: torch.Tensor | None = None
    src_type: GGMLType | None = None
    tiled: torch.Tensor | None = None  # device layout (built on first use; planes then dropped)

    @property
    def device(self) -> torch.device:
        return (self.tiled if self.tiled is not None else self.p0).device

    def nbytes(self) -> int:
        if self.tiled is not None:
            return self.tiled.numel()
        return sum(t.numel() * t.element_size() for t in (self.p0, self.p1, self.p2, self.d) if t is not None)

    def finalize(self) -> "QWeight":
        """Build the tiled device layout and release the planar planes."""
        if self.wtype != W_BF16 and self.tiled is None:
            self.tiled = tile_planes(self)
            self.p0 = self.p1 = self.p2 = self.d = None
        return self

    def _planar(self) -> "QWeight":
        if self.tiled is not None:  # rebuild planes (row operations after tiling)
            pl = untile_planes(self)
            return QWeight(self.wtype, self.N, self.K, pl["p0"], pl.get("p1"), pl.get("p2"), pl.get("d"), self.src_type)
        return self

    def args(self):
        if self.wtype == W_BF16:
            return (self.wtype, self.N, self.K, self.p0, None, None, None)
        self.finalize()
        return (self.wtype, self.N, self.K, self.tiled, None, None, None)

    @staticmethod
    def from_packed(raw: torch.Tensor, t: GGMLType, N: int, K: int, device=None) -> "QWeight":
        """raw: uint8 ``[N, row_bytes]`` GGUF rows (any device)."""
        t = GGMLType(t)
        dev = torch.device(device) if device is not None else raw.device
        raw = raw.to(dev)
        if t in IK_TYPES:  # ik_llama row-scaled type: requantize to a type the kernels stream
            from ..models.weights import import_ik

            tt, q = import_ik(raw.cpu().numpy(), t, (N, K), dev)
            return QWeight.from_packed(q, tt, N, K, dev)
        if t == GGMLType.Q3_K and K % 256 == 0:  # exact: same super-block structure as Q6_K
            return QWeight.from_packed(q3_k_as_q6_k(raw, N, K), GGMLType.Q6_K, N, K, dev)
        if t == GGMLType.IQ4_XS and K % 256 == 0:  # same codes, per-block fp16 scales
            return QWeight.from_packed(iq4_xs_as_iq4_nl(raw, N, K), GGMLType.IQ4_NL, N, K, dev)
        if t not in NATIVE and t in _REQUANT and K % 64 == 0:
            # block types without a tiled kernel format (Q5_0, Q2_K, Q4_1, ...): import as Q8_0,
            # which the GEMV / tcgen05 GEMM stream (exact for Q5_0, near-lossless otherwise)
            return QWeight.from_packed(requant_q8_0(raw, t, N, K), GGMLType.Q8_0, N, K, dev)
        if t not in NATIVE or K % TILE_FMT[int(t)][0]:
            if t == GGMLType.BF16:
                w = raw.contiguous().view(torch.bfloat16).reshape(N, K)
            elif t == GGMLType.F16:
                w = raw.contiguous().view(torch.float16).reshape(N, K).to(torch.bfloat16)
            elif t == GGMLType.F32:
                w = raw.contiguous().view(torch.float32).reshape(N, K).to(torch.bfloat16)
            else:
                arr = dequantize(raw.cpu().numpy(), t, (N, K))
                w = torch.from_numpy(arr).to(dev, torch.bfloat16)
            return QWeight(W_BF16, N, K, w.contiguous().view(torch.uint8), src_type=t)
        b = _blocks(raw, N, t)
        c = lambda x: x.contiguous().reshape(N, -1)  # noqa: E731
        if t in (GGMLType.Q4_0, GGMLType.IQ4_NL):
            return QWeight(int(t), N, K, c(b[..., 2:18]), d=_u16(b[..., 0:2]).reshape(N, -1).contiguous(), src_type=t)
        if t == GGMLType.Q8_0:
            return QWeight(int(t), N, K, c(b[..., 2:34]), d=_u16(b[..., 0:2]).reshape(N, -1).contiguous(), src_type=t)
        if t == GGMLType.Q4_K:
            return QWeight(int(t), N, K, c(b[..., 16:144]), p2=c(b[..., 0:16]), src_type=t)
        if t == GGMLType.Q5_K:
            return QWeight(int(t), N, K, c(b[..., 48:176]), p1=c(b[..., 16:48]), p2=c(b[..., 0:16]), src_type=t)
        if t == GGMLType.Q6_K:
            return QWeight(int(t), N, K, c(b[..., 0:128]), p1=c(b[..., 128:192]), p2=c(b[..., 192:208]),
                           d=_u16(b[..., 208:210]).reshape(N, -1).contiguous(), src_type=t)
        raise AssertionError(t)

    def to_gguf_rows(self) -> torch.Tensor:
        """Inverse of ``from_packed`` (and of the tiling) for native types: uint8 ``[N, row_bytes]``."""
        self = self._planar()
        t = GGMLType(self.wtype)
        N = self.N
        nbk = lambda x, per: x.reshape(N, -1, per)  # noqa: E731
        dd = lambda: self.d.contiguous().view(torch.uint8).reshape(N, -1, 2)  # noqa: E731
        if t in (GGMLType.Q4_0, GGMLType.IQ4_NL):
            parts = [dd(), nbk(self.p0, 16)]
        elif t == GGMLType.Q8_0:
            parts = [dd(), nbk(self.p0, 32)]
        elif t == GGMLType.Q4_K:
            parts = [nbk(self.p2, 16), nbk(self.p0, 128)]
        elif t == GGMLType.Q5_K:
            parts = [nbk(self.p2, 16), nbk(self.p1, 32), nbk(self.p0, 128)]
        elif t == GGMLType.Q6_K:
            parts = [nbk(self.p0, 128), nbk(self.p1, 64), nbk(self.p2, 16), dd()]
        else:
            raise ValueError("bf16 weights have no GGUF block form")
        return torch.cat(parts, -1).reshape(N, -1)

    def select_rows(self, idx: torch.Tensor) -> "QWeight":
        """Row gather (used to fuse/interleave projections and to shard for tensor parallelism)."""
        self = self._planar()
        idx = idx.to(self.p0.device)
        g = lambda x: None if x is None else x.index_select(0, idx).contiguous()  # noqa: E731
        return QWeight(self.wtype, int(idx.numel()), self.K, g(self.p0), g(self.p1), g(self.p2), g(self.d), self.src_type)

    def row_slice(self, r0: int, n: int) -> "QWeight":
        """Rows [r0, r0+n) as a view of the tiled buffer (r0, n multiples of 128), e.g. one expert of a
        stacked expert tensor."""
        if self.wtype == W_BF16:
            return QWeight(W_BF16, n, self.K, self.p0[r0:r0 + n], None, None, None, self.src_type)
        if r0 % 128 or n % 128:
            raise ValueError("row_slice: rows must be multiples of 128")
        self.finalize()
        G, _ = TILE_FMT[self.wtype]
        per_tile = self.tiled.numel() // ((self.N + 127) // 128)
        q = QWeight(self.wtype, n, self.K, None, None, None, None, self.src_type)
        q.tiled = self.tiled[(r0 // 128) * per_tile:(r0 + n) // 128 * per_tile]
        return q

    def col_shard(self, k0: int, k1: int) -> "QWeight":
        """Columns [k0, k1) (block-aligned) — row-parallel sharding for tensor parallelism."""
        self = self._planar()
        K = self.K
        bs = 256 if self.wtype in (12, 13, 14) else (32 if self.wtype else 1)
        if k0 % bs or k1 % bs:
            raise ValueError(f"column shard [{k0},{k1}) not aligned to block {bs}")
        def cs(x):
            if x is None:
                return None
            per = x.shape[1] * (1 if x.dim() == 2 else 1)
            a, b = k0 * per // K, k1 * per // K
            return x[:, a:b].contiguous()
        return QWeight(self.wtype, self.N, k1 - k0, cs(self.p0), cs(self.p1), cs(self.p2), cs(self.d), self.src_type)


# ---------------------------------------------------------------- tiled device layout (qtile.cuh)
# per type: group size G and planes in chunk order as (planar attribute, bytes per group per row)
TILE_FMT = {
    int(GGMLType.Q4_K): (256, [("p0", 128), ("p2", 16)]),
    int(GGMLType.Q5_K): (256, [("p0", 128), ("p1", 32), ("p2", 16)]),
    int(GGMLType.Q6_K): (256, [("p0", 128), ("p1", 64), ("p2", 16), ("d", 2)]),
    int(GGMLType.Q8_0): (64, [("p0", 64), ("d", 4)]),
    int(GGMLType.Q4_0): (64, [("p0", 32), ("d", 4)]),
    int(GGMLType.IQ4_NL): (64, [("p0", 32), ("d", 4)]),
}


def _swz_index(rb: int, device) -> torch.Tensor | None:
    """[128, rb/16] physical->logical chunk map (XOR swizzle is its own inverse)."""
    if rb not in (32, 64, 128):
        return None
    r = torch.arange(128, device=device)[:, None]
    c = torch.arange(rb // 16, device=device)[None, :]
    f = {128: r & 7, 64: (r >> 1) & 3, 32: (r >> 2) & 1}[rb]
    return c ^ f


def tile_planes(w: "QWeight") -> torch.Tensor:
    """Planar planes -> one uint8 buffer of chunks [NT, KG, CHUNK] (rows padded to 128)."""
    G, planes = TILE_FMT[w.wtype]
    N, K = w.N, w.K
    NT, KG = (N + 127) // 128, K // G
    parts = []
    for attr, rb in planes:
        x = getattr(w, attr)
        x = x.contiguous().view(torch.uint8).reshape(N, KG, rb)
        if NT * 128 != N:
            x = torch.cat([x, torch.zeros(NT * 128 - N, KG, rb, dtype=torch.uint8, device=x.device)], 0)
        x = x.reshape(NT, 128, KG, rb)
        idx = _swz_index(rb, x.device)
        if idx is not None:
            x = x.reshape(NT, 128, KG, rb // 16, 16)
            g = idx[None, :, None, :, None].expand(NT, 128, KG, rb // 16, 16)
            x = torch.gather(x, 3, g).reshape(NT, 128, KG, rb)
        parts.append(x.permute(0, 2, 1, 3).reshape(NT, KG, 128 * rb))
    return torch.cat(parts, -1).contiguous().reshape(-1)


def untile_planes(w: "QWeight") -> dict:
    """Inverse of ``tile_planes``: tiled buffer -> planar planes (same attributes as before)."""
    G, planes = TILE_FMT[w.wtype]
    N, K = w.N, w.K
    NT, KG = (N + 127) // 128, K // G
    buf = w.tiled.reshape(NT, KG, -1)
    out, off = {}, 0
    for attr, rb in planes:
        x = buf[:, :, off:off + 128 * rb].reshape(NT, KG, 128, rb).permute(0, 2, 1, 3)
        off += 128 * rb
        idx = _swz_index(rb, x.device)
        if idx is not None:
            x = x.reshape(NT, 128, KG, rb // 16, 16)
            g = idx[None, :, None, :, None].expand(NT, 128, KG, rb // 16, 16)
            x = torch.gather(x, 3, g)
        x = x.reshape(NT * 128, KG * rb)[:N].contiguous()
        out[attr] = x.view(torch.int16) if attr == "d" else x
    return out


def cat_rows(ws: list[QWeight]) -> QWeight:
    ws = [w._planar() for w in ws]
    t = ws[0].wtype
    if any(w.wtype != t or w.K != ws[0].K for w in ws):
        raise ValueError("cat_rows: types or K differ")
    c = lambda xs: None if xs[0] is None else torch.cat(xs, 0)  # noqa: E731
    return QWeight(t, sum(w.N for w in ws), ws[0].K, c([w.p0 for w in ws]), c([w.p1 for w in ws]),
                   c([w.p2 for w in ws]), c([w.d for w in ws]), ws[0].src_type)


def interleave_gate_up(gate: QWeight, up: QWeight, group: int = 32) -> QWeight:
    """Rows ordered [gate 32g..32g+31, up 32g..32g+31] per group (the SwiGLU epilogues' layout)."""
    if gate.N != up.N or gate.N % group:
        raise ValueError("interleave_gate_up: N must match and be a multiple of the group")
    both = cat_rows([gate, up])
    F = gate.N
    g = torch.arange(F).view(F // group, 1, group)
    idx = torch.cat([g, g + F], 1).reshape(-1)
    return both.select_rows(idx)
