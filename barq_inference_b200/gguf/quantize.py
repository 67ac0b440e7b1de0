"""Vectorized ggml-layout quantizers in PyTorch (run on CPU or on the GPU).

They write the standard GGUF block layouts bit-exactly (the NumPy dequantizers in
``dequant.py`` read them back).  Scale search is simpler than ggml's iterative
``make_qkx2_quants``: per-sub-block min/max (K-quants) or absmax (symmetric types)
followed by 6/8-bit scale quantization.  That is enough for ``convert`` and for the
random-init benchmark checkpoints; the reference's own quantizers write private
layouts instead (``quant/src/q4_0.rs:9,59-63``, ``quant/src/q4_k.rs:65-72``).

All functions take ``x`` with last dim a multiple of the block size and return a
``uint8`` tensor of shape ``x.shape[:-1] + (row_bytes,)``.
"""
from __future__ import annotations

import torch

from .constants import KVALUES_IQ4NL, QK_K, TYPE_TRAITS, GGMLType


def _f16_bytes(v: torch.Tensor) -> torch.Tensor:
    """[..., 1] float -> [..., 2] uint8 little-endian fp16."""
    return v.to(torch.float16).contiguous().view(torch.uint8)


def _f16r(v: torch.Tensor) -> torch.Tensor:
    return v.to(torch.float16).to(torch.float32)


def _rows(x: torch.Tensor, bs: int) -> tuple[torch.Tensor, tuple[int, ...]]:
    if x.shape[-1] % bs:
        raise ValueError(f"last dim {x.shape[-1]} not a multiple of {bs}")
    lead = tuple(x.shape[:-1])
    return x.reshape(-1, bs).to(torch.float32), lead


def _finish(blocks: torch.Tensor, lead: tuple[int, ...], k: int, t: GGMLType) -> torch.Tensor:
    tr = TYPE_TRAITS[t]
    return blocks.reshape(*lead, k // tr.block_size * tr.type_size)


def _pack_nibbles(lo: torch.Tensor, hi: torch.Tensor) -> torch.Tensor:
    return (lo.to(torch.uint8) & 0xF) | ((hi.to(torch.uint8) & 0xF) << 4)


def _signed_absmax(x: torch.Tensor) -> torch.Tensor:
    idx = x.abs().argmax(dim=-1, keepdim=True)
    return torch.gather(x, -1, idx)


def quantize_q8_0(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    b, lead = _rows(x, 32)
    amax = b.abs().amax(-1, keepdim=True)
    d = amax / 127.0
    idv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    q = torch.round(b * idv).clamp(-127, 127).to(torch.int8)
    out = torch.cat([_f16_bytes(d), q.view(torch.uint8)], -1)
    return _finish(out, lead, k, GGMLType.Q8_0)


def quantize_q4_0(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    b, lead = _rows(x, 32)
    mx = _signed_absmax(b)
    d = mx / -8.0
    idv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    q = torch.clamp(torch.trunc(b * idv + 8.5), 0, 15).to(torch.uint8)
    qs = _pack_nibbles(q[:, :16], q[:, 16:])
    return _finish(torch.cat([_f16_bytes(d), qs], -1), lead, k, GGMLType.Q4_0)


def quantize_q4_1(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    b, lead = _rows(x, 32)
    mn = b.amin(-1, keepdim=True)
    mx = b.amax(-1, keepdim=True)
    d = (mx - mn) / 15.0
    idv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    q = torch.clamp(torch.trunc((b - mn) * idv + 0.5), 0, 15).to(torch.uint8)
    qs = _pack_nibbles(q[:, :16], q[:, 16:])
    return _finish(torch.cat([_f16_bytes(d), _f16_bytes(mn), qs], -1), lead, k, GGMLType.Q4_1)


def _qh_bits(q: torch.Tensor) -> torch.Tensor:
    """q: [nb, 32] 5-bit values -> [nb, 4] bytes of the 32 high bits (bit j = q[j] >> 4)."""
    hb = ((q.to(torch.int64) >> 4) & 1) << torch.arange(32, device=q.device, dtype=torch.int64)
    v = hb.sum(-1, keepdim=True)
    sh = torch.tensor([0, 8, 16, 24], device=q.device, dtype=torch.int64)
    return ((v >> sh) & 0xFF).to(torch.uint8)


def quantize_q5_0(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    b, lead = _rows(x, 32)
    mx = _signed_absmax(b)
    d = mx / -16.0
    idv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    q = torch.clamp(torch.trunc(b * idv + 16.5), 0, 31).to(torch.uint8)
    qs = _pack_nibbles(q[:, :16], q[:, 16:])
    return _finish(torch.cat([_f16_bytes(d), _qh_bits(q), qs], -1), lead, k, GGMLType.Q5_0)


def quantize_q5_1(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    b, lead = _rows(x, 32)
    mn = b.amin(-1, keepdim=True)
    mx = b.amax(-1, keepdim=True)
    d = (mx - mn) / 31.0
    idv = torch.where(d > 0, 1.0 / d, torch.zeros_like(d))
    q = torch.clamp(torch.trunc((b - mn) * idv + 0.5), 0, 31).to(torch.uint8)
    qs = _pack_nibbles(q[:, :16], q[:, 16:])
    return _finish(torch.cat([_f16_bytes(d), _f16_bytes(mn), _qh_bits(q), qs], -1), lead, k, GGMLType.Q5_1)


def _pack_k_scales(ls: torch.Tensor, lm: torch.Tensor) -> torch.Tensor:
    """6-bit (scale, min) x 8 -> the 12-byte K-quant scale field (inverse of get_scale_min_k4)."""
    ls = ls.to(torch.int32)
    lm = lm.to(torch.int32)
    out = torch.empty(ls.shape[0], 12, dtype=torch.int32, device=ls.device)
    out[:, 0:4] = (ls[:, 0:4] & 63) | ((ls[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (lm[:, 0:4] & 63) | ((lm[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (ls[:, 4:8] & 0xF) | ((lm[:, 4:8] & 0xF) << 4)
    return out.to(torch.uint8)


def _kquant_affine(b: torch.Tensor, nlev: int):
    """b: [nb, 256] -> (d16, dmin16, ls[nb,8], lm[nb,8], q[nb,256]) for Q4_K/Q5_K."""
    sb = b.reshape(-1, 8, 32)
    mn = sb.amin(-1).clamp(max=0.0)
    mx = sb.amax(-1)
    scale = (mx - mn) / nlev
    minv = -mn
    d = _f16r(scale.amax(-1, keepdim=True) / 63.0)
    dmin = _f16r(minv.amax(-1, keepdim=True) / 63.0)
    ls = torch.where(d > 0, torch.round(scale / d.clamp_min(1e-30)), torch.zeros_like(scale)).clamp(0, 63)
    lm = torch.where(dmin > 0, torch.round(minv / dmin.clamp_min(1e-30)), torch.zeros_like(minv)).clamp(0, 63)
    eff_d = (d * ls).unsqueeze(-1)
    eff_m = (dmin * lm).unsqueeze(-1)
    q = torch.where(eff_d > 0, torch.round((sb + eff_m) / eff_d.clamp_min(1e-30)), torch.zeros_like(sb)).clamp(0, nlev)
    return d, dmin, ls, lm, q.reshape(-1, 256).to(torch.int32)


def quantize_q4_k(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    b, lead = _rows(x, QK_K)
    d, dmin, ls, lm, q = _kquant_affine(b, 15)
    qv = q.reshape(-1, 4, 2, 32)
    qs = _pack_nibbles(qv[:, :, 0, :], qv[:, :, 1, :]).reshape(-1, 128)
    out = torch.cat([_f16_bytes(d), _f16_bytes(dmin), _pack_k_scales(ls, lm), qs], -1)
    return _finish(out, lead, k, GGMLType.Q4_K)


def quantize_q5_k(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    b, lead = _rows(x, QK_K)
    d, dmin, ls, lm, q = _kquant_affine(b, 31)
    qv = q.reshape(-1, 4, 2, 32)
    ql = _pack_nibbles(qv[:, :, 0, :] & 0xF, qv[:, :, 1, :] & 0xF).reshape(-1, 128)
    hi = (qv >> 4) & 1  # [nb, 4(j), 2(half), 32(l)] -> bit (2j + half) of qh[l]
    sh = (2 * torch.arange(4, device=x.device).view(1, 4, 1, 1) + torch.arange(2, device=x.device).view(1, 1, 2, 1))
    qh = (hi << sh).sum(dim=(1, 2)).to(torch.uint8)
    out = torch.cat([_f16_bytes(d), _f16_bytes(dmin), _pack_k_scales(ls, lm), qh, ql], -1)
    return _finish(out, lead, k, GGMLType.Q5_K)


def quantize_q6_k(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    b, lead = _rows(x, QK_K)
    sb = b.reshape(-1, 16, 16)
    mx = _signed_absmax(sb).squeeze(-1)  # [nb,16]
    scale = mx / -32.0
    dmax = _signed_absmax(scale)  # [nb,1]
    d = _f16r(dmax / -128.0)
    sc = torch.where(d != 0, torch.round(scale / torch.where(d != 0, d, torch.ones_like(d))), torch.zeros_like(scale)).clamp(-128, 127)
    eff = (d * sc).unsqueeze(-1)
    q = torch.where(eff != 0, torch.round(sb / torch.where(eff != 0, eff, torch.ones_like(eff))), torch.zeros_like(sb)).clamp(-32, 31)
    q = (q + 32).to(torch.int32).reshape(-1, 2, 4, 32)  # [nb, n, k(quarter), l]
    q1, q2, q3, q4 = q[:, :, 0], q[:, :, 1], q[:, :, 2], q[:, :, 3]
    ql = torch.cat([(q1 & 0xF) | ((q3 & 0xF) << 4), (q2 & 0xF) | ((q4 & 0xF) << 4)], -1).to(torch.uint8).reshape(-1, 128)
    qh = ((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)).to(torch.uint8).reshape(-1, 64)
    sc8 = sc.to(torch.int8).view(torch.uint8)
    out = torch.cat([ql, qh, sc8, _f16_bytes(d)], -1)
    return _finish(out, lead, k, GGMLType.Q6_K)


def quantize_iq4_nl(x: torch.Tensor) -> torch.Tensor:
    k = x.shape[-1]
    b, lead = _rows(x, 32)
    kv = torch.tensor(KVALUES_IQ4NL, dtype=torch.float32, device=b.device)
    mx = _signed_absmax(b)
    d0 = mx / kv[0]
    idv = torch.where(d0 != 0, 1.0 / d0, torch.zeros_like(d0))
    idx = (b * idv).unsqueeze(-1).sub(kv).abs().argmin(-1)
    qv = kv[idx]
    sumqx = (b * qv).sum(-1, keepdim=True)
    sumq2 = (qv * qv).sum(-1, keepdim=True)
    d = torch.where(sumq2 > 0, sumqx / sumq2, d0)
    qs = _pack_nibbles(idx[:, :16], idx[:, 16:])
    return _finish(torch.cat([_f16_bytes(d), qs], -1), lead, k, GGMLType.IQ4_NL)


def quantize_bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).contiguous().view(torch.uint8)


def quantize_f16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.float16).contiguous().view(torch.uint8)


def quantize_f32(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.float32).contiguous().view(torch.uint8)


QUANTIZERS = {
    GGMLType.F32: quantize_f32,
    GGMLType.F16: quantize_f16,
    GGMLType.BF16: quantize_bf16,
    GGMLType.Q4_0: quantize_q4_0,
    GGMLType.Q4_1: quantize_q4_1,
    GGMLType.Q5_0: quantize_q5_0,
    GGMLType.Q5_1: quantize_q5_1,
    GGMLType.Q8_0: quantize_q8_0,
    GGMLType.Q4_K: quantize_q4_k,
    GGMLType.Q5_K: quantize_q5_k,
    GGMLType.Q6_K: quantize_q6_k,
    GGMLType.IQ4_NL: quantize_iq4_nl,
}


def _ik_quantizers():
    from .ik_quants import Q_IK

    QUANTIZERS.update(Q_IK)


def _ternary(name: str):
    """TQ1_0 / TQ2_0 quantizers (numpy, ``gguf/ternary.py``) with the torch signature used here:
    [..., K] float -> [..., row bytes] uint8."""
    def q(x: torch.Tensor) -> torch.Tensor:
        from . import ternary

        k = x.shape[-1]
        if k % 256:
            raise ValueError(f"{name}: row length {k} is not a multiple of 256")
        lead = x.shape[:-1]
        packed = getattr(ternary, name)(x.detach().float().cpu().numpy().reshape(-1, k))
        return torch.from_numpy(packed.reshape(*lead, -1)).to(x.device)
    return q


QUANTIZERS[GGMLType.TQ1_0] = _ternary("q_tq1_0")
QUANTIZERS[GGMLType.TQ2_0] = _ternary("q_tq2_0")


_ik_quantizers()


def quantize(x: torch.Tensor, t: GGMLType) -> torch.Tensor:
    t = GGMLType(t)
    if t not in QUANTIZERS:
        raise NotImplementedError(f"quantize: {t.name}")
    return QUANTIZERS[t](x)
