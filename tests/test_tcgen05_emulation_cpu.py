"""CPU check of the tcgen05 prefill attention kernel (``prefill_attn_tc_kernel`` in
``csrc/kernels/attn_prefill_tc.cu``) by emulating its data flow with ``tests/tcgen05_emu.py``: the
kernel's own shared-memory offsets (Q written with the 128-byte swizzle, K / V pages landed by TMA
boxes {64, 16}), UMMA descriptors (K-major Q and K, MN-major V), TMEM column plan (two S buffers,
P packed over the S columns it replaces, O at column 256), lazy-rescaled log2-domain softmax and
epilogue must reproduce fp32 causal / sliding-window attention over a paged cache.

The emulator itself is first checked on the tcgen05 GEMM's addressing (``csrc/kernels/gemm_tc.cu``:
swizzled weight writes or TMEM weight operands, TMA activation boxes, descriptors advanced by 32
bytes per 16-element step), whose results are verified on B200s: it must compute A B^T exactly.
"""
import numpy as np
import pytest

from tcgen05_emu import (IDESC_B_MAJOR_MN, Smem, Tmem, from_bits, idesc_bf16, idesc_f16, mma, to_bits,
                         umma_desc_sw128, umma_desc_sw128_mn)


@pytest.mark.parametrize("ts", [False, True])
def test_emulator_reproduces_the_gemm_tile(ts):
    """GEMM stage layout with KS = 2 atoms (128 K values) and a 64-token tile, SS and TS forms."""
    rng = np.random.default_rng(1)
    BN, KS = 64, 2
    A_ATOM, B_ATOM = 128 * 128, BN * 128
    OFF_A, OFF_B = 0, KS * A_ATOM
    w = rng.standard_normal((128, 64 * KS)).astype(np.float32)
    x = rng.standard_normal((BN, 64 * KS)).astype(np.float32)
    wb, xb = to_bits(w, "bf16"), to_bits(x, "bf16")
    sm, tm = Smem(), Tmem()
    ACOL = 2 * 2 * BN  # Issuers<64>: two issuers, two buffers
    for a in range(KS):
        sm.tma_2d_sw128(OFF_B + a * B_ATOM, xb[:, 64 * a: 64 * a + 64])  # activation box {64, BN}
        for qq in range(4):  # 16-element group qq of atom a, written by dequant warp quarter qq
            ops = wb[:, 64 * a + 16 * qq: 64 * a + 16 * qq + 16]
            if ts:  # tmem_st8(ta + a * 32) with ta = ACOL + qq * 8 (stage 0)
                words = ops[:, 0::2].astype(np.uint32) | (ops[:, 1::2].astype(np.uint32) << 16)
                tm.st_u32(0, ACOL + a * 32 + qq * 8, words)
                continue
            for half in range(2):
                r = np.arange(128)
                chunk = (2 * qq + half) ^ (r & 7)
                for e in range(8):
                    sm.store16(OFF_A + a * A_ATOM + r * 128 + chunk * 16 + 2 * e, ops[:, 8 * half + e])
    idesc = idesc_bf16(128, BN)
    for a in range(KS):
        for k in range(4):
            b = umma_desc_sw128(OFF_B + a * B_ATOM + 32 * k)
            if ts:
                mma(tm, 0, ACOL + a * 32 + k * 8, b, idesc, bool(a | k), sm, a_tmem=True)
            else:
                mma(tm, 0, umma_desc_sw128(OFF_A + a * A_ATOM + 32 * k), b, idesc, bool(a | k), sm)
    got = tm.w[:, :BN].view(np.float32).astype(np.float64)
    ref = from_bits(wb, "bf16") @ from_bits(xb, "bf16").T
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)


def test_mn_major_descriptor_reads_tma_rows_transposed():
    """A [keys, D] TMA tile read through the MN-major descriptor is B[n = d][k = key]."""
    rng = np.random.default_rng(2)
    keys, D = 128, 128
    v = to_bits(rng.standard_normal((keys, D)), "bf16")
    sm = Smem()
    ATOM = 128 * 128
    for p in range(keys // 16):  # page boxes as the producer lands them
        for at in range(D // 64):
            sm.tma_2d_sw128(at * ATOM + p * 2048, v[16 * p: 16 * p + 16, 64 * at: 64 * at + 64])
    from tcgen05_emu import read_operand
    for kk in range(keys // 16):
        B = read_operand(sm, umma_desc_sw128_mn(kk * 2048, ATOM), D, True, "bf16")
        np.testing.assert_array_equal(B, from_bits(v[16 * kk: 16 * kk + 16], "bf16").T)


# ---------------------------------------------------------------------------- the attention kernel
ROWS, KEYS, OCOL, RESCALE = 128, 128, 256, 8.0


def emulate_prefill_tc(q, kc, vc, bt, q_start, ctx_lens, H, Hkv, D, scale, window, dtype):
    """prefill_attn_tc_kernel, one CTA at a time, roles run in the order their barriers allow."""
    ATOMS, ATOM = D // 64, 128 * 128
    TILE = ATOMS * ATOM
    OFF_Q, OFF_K = 0, TILE
    OFF_V = OFF_K + 2 * TILE
    S = len(ctx_lens)
    G = H // Hkv
    T = q.shape[0]
    out = np.full((T, H, D), np.nan)
    nblk = kc.shape[0]
    k2d = to_bits(kc.reshape(nblk * Hkv * 16, D), dtype)
    v2d = to_bits(vc.reshape(nblk * Hkv * 16, D), dtype)
    qbits = to_bits(from_bits(to_bits(q, "bf16"), "bf16"), dtype)  # q is bf16; fp16 caches convert it
    sl2 = scale * 1.4426950408889634
    id_s = (idesc_f16 if dtype == "fp16" else idesc_bf16)(128, KEYS)
    id_o = (idesc_f16 if dtype == "fp16" else idesc_bf16)(128, D) | IDESC_B_MAJOR_MN
    max_q = max(q_start[i + 1] - q_start[i] for i in range(S))
    for s in range(S):
        q_begin, n_new = q_start[s], q_start[s + 1] - q_start[s]
        for h in range(H):
            for qt in range((max_q + ROWS - 1) // ROWS):
                q0 = qt * ROWS
                if q0 >= n_new:
                    continue
                ctx = ctx_lens[s]
                base_pos, kvh = ctx - n_new, h // G
                q_last = min(q0 + ROWS, n_new) - 1
                kv_end = base_pos + q_last + 1
                kv_begin = max(0, base_pos + q0 - window + 1) if window > 0 else 0
                t_begin, t_end = kv_begin // KEYS, (kv_end + KEYS - 1) // KEYS
                nt = t_end - t_begin
                sm, tm = Smem(), Tmem()
                # Q rows -> swizzled K-major atoms
                r = np.arange(ROWS)
                qi = q0 + r
                for c in range(D // 8):
                    for e in range(8):
                        vals = np.where(qi < n_new, qbits[np.minimum(q_begin + qi, T - 1), h, c * 8 + e], 0)
                        sm.store16(OFF_Q + (c >> 3) * ATOM + r * 128 + (((c & 7) ^ (r & 7)) << 4) + 2 * e, vals)
                pg_last = (kv_end - 1) >> 4

                def produce(j):
                    st, t = j % 2, t_begin + j
                    for p in range(KEYS // 16):
                        phys = bt[s][min(t * (KEYS // 16) + p, pg_last)]
                        y = (phys * Hkv + kvh) * 16
                        for at in range(ATOMS):
                            sm.tma_2d_sw128(OFF_K + st * TILE + at * ATOM + p * 2048, k2d[y:y + 16, at * 64:at * 64 + 64])
                            sm.tma_2d_sw128(OFF_V + st * TILE + at * ATOM + p * 2048, v2d[y:y + 16, at * 64:at * 64 + 64])

                def issue_s(j):
                    st = j % 2
                    produce(j)
                    for ks in range(D // 16):
                        at, kk = ks >> 2, ks & 3
                        mma(tm, st * KEYS, umma_desc_sw128(OFF_Q + at * ATOM + 32 * kk),
                            umma_desc_sw128(OFF_K + st * TILE + at * ATOM + 32 * kk), id_s, ks > 0, sm)

                qpos = base_pos + qi
                hi = np.minimum(qpos + 1, kv_end)
                lo = np.maximum(0, qpos - window + 1) if window > 0 else np.zeros_like(qpos)
                m_use = np.full(ROWS, -np.inf)
                l = np.zeros(ROWS)
                issue_s(0)
                for j in range(nt):
                    if j + 1 < nt:
                        issue_s(j + 1)
                    st = j % 2
                    k0 = (t_begin + j) * KEYS
                    Srow = tm.w[:, st * KEYS: st * KEYS + KEYS].view(np.float32).astype(np.float64)
                    kp = k0 + np.arange(KEYS)
                    vis = (kp[None, :] >= lo[:, None]) & (kp[None, :] < hi[:, None])
                    mx = np.where(vis, Srow, -np.inf).max(axis=1) * sl2
                    m_new = np.maximum(m_use, mx)
                    with np.errstate(invalid="ignore"):
                        resc = m_new > m_use + RESCALE
                        f = np.where(resc, np.exp2(np.where(resc, m_use - m_new, 0.0)), 1.0)
                    if j > 0 and resc.any():
                        O = tm.w[:, OCOL:OCOL + D].view(np.float32).astype(np.float64) * f[:, None]
                        tm.w[:, OCOL:OCOL + D] = O.astype(np.float32).view(np.uint32)
                    l = np.where(resc, l * f, l)
                    m_use = np.where(resc, m_new, m_use)
                    with np.errstate(invalid="ignore", over="ignore"):
                        P = np.where(vis, np.exp2(Srow * sl2 - m_use[:, None]), 0.0)
                    l = l + P.sum(axis=1)
                    pb = to_bits(P, dtype).astype(np.uint32)
                    tm.w[:, st * KEYS: st * KEYS + KEYS // 2] = pb[:, 0::2] | (pb[:, 1::2] << 16)
                    for kk in range(KEYS // 16):
                        mma(tm, OCOL, st * KEYS + kk * 8, umma_desc_sw128_mn(OFF_V + st * TILE + kk * 2048, ATOM),
                            id_o, bool((j > 0) | (kk > 0)), sm, a_tmem=True)
                O = tm.w[:, OCOL:OCOL + D].view(np.float32).astype(np.float64)
                inv = np.where(l > 0, 1.0 / np.where(l > 0, l, 1.0), 0.0)
                for rr in range(ROWS):
                    if qi[rr] < n_new:
                        out[q_begin + qi[rr], h] = O[rr] * inv[rr]
    return out


def reference_attention(q, kc, vc, bt, q_start, ctx_lens, H, Hkv, D, scale, window):
    out = np.zeros((q.shape[0], H, D))
    G = H // Hkv
    for s in range(len(ctx_lens)):
        n_new, ctx = q_start[s + 1] - q_start[s], ctx_lens[s]
        pos = np.arange(ctx)
        K = kc[[bt[s][p >> 4] for p in pos], :, pos & 15]  # [ctx, Hkv, D]
        V = vc[[bt[s][p >> 4] for p in pos], :, pos & 15]
        for i in range(n_new):
            qp = ctx - n_new + i
            vis = (pos <= qp) & ((pos > qp - window) if window > 0 else True)
            for h in range(H):
                sc = K[:, h // G] @ q[q_start[s] + i, h] * scale
                sc = np.where(vis, sc, -np.inf)
                p = np.exp(sc - sc.max())
                out[q_start[s] + i, h] = p @ V[:, h // G] / p.sum()
    return out


@pytest.mark.parametrize("D,dtype,window", [(128, "bf16", 0), (64, "fp16", 0), (128, "fp16", 200), (64, "bf16", 37)])
def test_prefill_tc_dataflow_matches_fp32_attention(D, dtype, window):
    rng = np.random.default_rng(3 + D + window)
    H, Hkv = 4, 2
    # a first prefill (130 tokens, two query tiles) and a later chunk on top of a 300-token prefix
    seqs = [(130, 130), (70, 370)]
    nblk = 64
    perm = rng.permutation(nblk)
    bt, used = [], 0
    for _, ctx in seqs:
        n = (ctx + 15) // 16
        bt.append(list(perm[used:used + n]) + [0] * 2)
        used += n
    q_start = [0]
    for n, _ in seqs:
        q_start.append(q_start[-1] + n)
    T = q_start[-1]
    q = rng.standard_normal((T, H, D)).astype(np.float32) * 2.0  # large enough scores to exercise rescales
    kc = rng.standard_normal((nblk, Hkv, 16, D)).astype(np.float32)
    vc = rng.standard_normal((nblk, Hkv, 16, D)).astype(np.float32)
    # the kernel works on 16-bit operands: compare against fp32 attention of the same rounded values
    qr = from_bits(to_bits(q, "bf16"), "bf16")
    if dtype == "fp16":
        qr = from_bits(to_bits(qr, "fp16"), "fp16")
    kr, vr = from_bits(to_bits(kc, dtype), dtype), from_bits(to_bits(vc, dtype), dtype)
    ctx_lens = [c for _, c in seqs]
    scale = 1.0 / np.sqrt(D)
    got = emulate_prefill_tc(q, kc, vc, bt, q_start, ctx_lens, H, Hkv, D, scale, window, dtype)
    ref = reference_attention(qr, kr, vr, bt, q_start, ctx_lens, H, Hkv, D, scale, window)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    assert err < 2e-2, err
