"""CPU check of the tensor-core MLA decode kernel (``mla_attn_mma_kernel`` in ``csrc/kernels/mla.cu``)
by lane-level emulation (``tests/mma_emu.py``): the kernel's own fragment addresses, page split,
per-warp dimension slices, partial-score exchange, log2-domain online softmax, P packing and
natural-log partials, followed by the split merge, must reproduce fp32 absorbed MLA attention.

The emulator's fragment semantics are first checked on the addressing of the decode-attention
kernel (``csrc/kernels/attn_decode.cu``), whose results are verified on the GPU: with the same
ldmatrix row addresses, the modelled instructions must compute Q K^T and P V exactly.
"""
import numpy as np
import pytest

from mma_emu import G, LANE, T, ldsm_x4, mma, pack, round_to, shfl_xor_max, shfl_xor_sum

K_ROW, K_LAT, K_PAGE, H = 576, 512, 16, 16
LD = K_ROW + 8
NW, KSW, NDW, RING = 4, 9, 16, 4
LOG2E, LN2 = 1.4426950408889634, 0.6931471805599453


def test_emulator_reproduces_the_decode_kernel_products():
    """Decode-attention addressing (D = 128, rows padded to D + 8): Q K^T and P V are exact."""
    rng = np.random.default_rng(0)
    D, ld = 128, 136
    q = round_to(rng.standard_normal((16, D)), "bf16")
    k = round_to(rng.standard_normal((16, D)), "bf16")
    v = round_to(rng.standard_normal((16, D)), "bf16")
    sq, sk, sv = (np.zeros(16 * ld) for _ in range(3))
    for r in range(16):
        sq[r * ld: r * ld + D], sk[r * ld: r * ld + D], sv[r * ld: r * ld + D] = q[r], k[r], v[r]
    sc = np.zeros((2, 32, 4))
    for kk in range(D // 16):
        qf = ldsm_x4(sq, ((LANE & 7) + ((LANE >> 3) & 1) * 8) * ld + kk * 16 + (LANE >> 4) * 8)
        kf = ldsm_x4(sk, ((LANE & 7) + (LANE >> 4) * 8) * ld + kk * 16 + ((LANE >> 3) & 1) * 8)
        mma(sc[0], qf, kf[:, 0:2])
        mma(sc[1], qf, kf[:, 2:4])
    S = np.zeros((16, 16))
    for j in range(2):
        S[G, j * 8 + 2 * T], S[G, j * 8 + 2 * T + 1] = sc[j][:, 0], sc[j][:, 1]
        S[G + 8, j * 8 + 2 * T], S[G + 8, j * 8 + 2 * T + 1] = sc[j][:, 2], sc[j][:, 3]
    np.testing.assert_allclose(S, q @ k.T, rtol=1e-12, atol=1e-12)
    p = round_to(rng.random((16, 16)), "bf16")  # P as the A operand, laid out like the S fragments
    pf = np.stack([pack(p[G, 2 * T], p[G, 2 * T + 1], "bf16"), pack(p[G + 8, 2 * T], p[G + 8, 2 * T + 1], "bf16"),
                   pack(p[G, 8 + 2 * T], p[G, 9 + 2 * T], "bf16"), pack(p[G + 8, 8 + 2 * T], p[G + 8, 9 + 2 * T], "bf16")],
                  axis=1)
    o = np.zeros((D // 8, 32, 4))
    for jd in range(0, D // 8, 2):
        vf = ldsm_x4(sv, ((LANE & 7) + ((LANE >> 3) & 1) * 8) * ld + jd * 8 + (LANE >> 4) * 8, trans=True)
        mma(o[jd], pf, vf[:, 0:2])
        mma(o[jd + 1], pf, vf[:, 2:4])
    O = np.zeros((16, D))
    for jd in range(D // 8):
        O[G, jd * 8 + 2 * T], O[G, jd * 8 + 2 * T + 1] = o[jd][:, 0], o[jd][:, 1]
        O[G + 8, jd * 8 + 2 * T], O[G + 8, jd * 8 + 2 * T + 1] = o[jd][:, 2], o[jd][:, 3]
    np.testing.assert_allclose(O, p @ v, rtol=1e-12, atol=1e-12)


def emulate_mla_mma(q_lat, q_pe, cache, bt, row_seq, row_len, splits, scale, dtype):
    """The kernel (one CTA per (split, row), warps emulated in turn per page) plus mla_merge_kernel."""
    rows = q_lat.shape[0]
    part_acc = np.zeros((rows, splits, H, K_LAT))
    part_ml = np.zeros((rows, splits, H, 2))
    for row in range(rows):
        sQ = np.zeros(16 * LD)
        qfull = np.concatenate([q_lat[row], q_pe[row]], axis=1)  # [16, 576]
        for h in range(H):
            sQ[h * LD: h * LD + K_ROW] = round_to(qfull[h] * np.float32(scale), dtype)
        seq, ln = int(row_seq[row]), int(row_len[row])
        npages = (ln + K_PAGE - 1) // K_PAGE
        per = (npages + splits - 1) // splits
        for split in range(splits):
            pb = split * per
            npg = max(0, min(npages, pb + per) - pb)
            ring = np.zeros(RING * K_PAGE * LD)
            qf = [[ldsm_x4(sQ, ((LANE & 7) + ((LANE >> 3) & 1) * 8) * LD + (w * KSW + kk) * 16 + (LANE >> 4) * 8)
                   for kk in range(KSW)] for w in range(NW)]
            o = np.zeros((NW, NDW, 32, 4))
            m0, m1 = np.full((NW, 32), -1e30), np.full((NW, 32), -1e30)
            l0, l1 = np.zeros((NW, 32)), np.zeros((NW, 32))
            sx = np.zeros((2, NW, 256))
            for i in range(npg):
                s = i % RING
                phys = int(bt[seq, pb + i])
                base = s * K_PAGE * LD
                for r in range(K_PAGE):  # the copy warp's pieces land in the padded rows
                    ring[base + r * LD: base + r * LD + K_ROW] = cache[phys, r]
                for w in range(NW):  # partial scores of each warp's 144 dims
                    sc = np.zeros((2, 32, 4))
                    for kk in range(KSW):
                        addr = base + ((LANE & 7) + (LANE >> 4) * 8) * LD + (w * KSW + kk) * 16 + ((LANE >> 3) & 1) * 8
                        kf = ldsm_x4(ring, addr)
                        mma(sc[0], qf[w][kk], kf[:, 0:2])
                        mma(sc[1], qf[w][kk], kf[:, 2:4])
                    xw = sx[i & 1, w]
                    for j in range(2):
                        xw[G * 16 + j * 8 + 2 * T], xw[G * 16 + j * 8 + 2 * T + 1] = sc[j][:, 0], sc[j][:, 1]
                        xw[(G + 8) * 16 + j * 8 + 2 * T], xw[(G + 8) * 16 + j * 8 + 2 * T + 1] = sc[j][:, 2], sc[j][:, 3]
                for w in range(NW):  # after the named barrier
                    x0 = sx[i & 1]
                    sc = np.zeros((2, 32, 4))
                    for j in range(2):
                        for hh in range(2):
                            off = (G + 8 * hh) * 16 + j * 8 + 2 * T
                            vx, vy = x0[0][off].copy(), x0[0][off + 1].copy()
                            for ww in range(1, NW):
                                vx, vy = vx + x0[ww][off], vy + x0[ww][off + 1]
                            sc[j][:, 2 * hh], sc[j][:, 2 * hh + 1] = vx, vy
                    mn0, mn1 = m0[w].copy(), m1[w].copy()
                    for j in range(2):
                        for e in range(4):
                            tok = (pb + i) * K_PAGE + j * 8 + 2 * T + (e & 1)
                            v = np.where(tok < ln, sc[j][:, e] * LOG2E, -np.inf)
                            sc[j][:, e] = v
                            if e < 2:
                                mn0 = np.maximum(mn0, v)
                            else:
                                mn1 = np.maximum(mn1, v)
                    mn0, mn1 = shfl_xor_max(mn0), shfl_xor_max(mn1)
                    c0, c1 = np.exp2(m0[w] - mn0), np.exp2(m1[w] - mn1)
                    ps0, ps1 = np.zeros(32), np.zeros(32)
                    for j in range(2):
                        for e in range(4):
                            p = np.exp2(sc[j][:, e] - (mn0 if e < 2 else mn1))
                            sc[j][:, e] = p
                            if e < 2:
                                ps0 += p
                            else:
                                ps1 += p
                    ps0, ps1 = shfl_xor_sum(ps0), shfl_xor_sum(ps1)
                    l0[w], l1[w] = l0[w] * c0 + ps0, l1[w] * c1 + ps1
                    m0[w], m1[w] = mn0, mn1
                    o[w][:, :, 0:2] *= c0[None, :, None]
                    o[w][:, :, 2:4] *= c1[None, :, None]
                    pf = np.stack([pack(sc[0][:, 0], sc[0][:, 1], dtype), pack(sc[0][:, 2], sc[0][:, 3], dtype),
                                   pack(sc[1][:, 0], sc[1][:, 1], dtype), pack(sc[1][:, 2], sc[1][:, 3], dtype)], axis=1)
                    for jd in range(0, NDW, 2):
                        addr = base + ((LANE & 7) + ((LANE >> 3) & 1) * 8) * LD + w * (K_LAT // NW) + jd * 8 + (LANE >> 4) * 8
                        vf = ldsm_x4(ring, addr, trans=True)
                        mma(o[w][jd], pf, vf[:, 0:2])
                        mma(o[w][jd + 1], pf, vf[:, 2:4])
            for w in range(NW):
                for jd in range(NDW):
                    d = w * (K_LAT // NW) + jd * 8 + 2 * T
                    part_acc[row, split, G, d], part_acc[row, split, G, d + 1] = o[w][jd][:, 0], o[w][jd][:, 1]
                    part_acc[row, split, G + 8, d], part_acc[row, split, G + 8, d + 1] = o[w][jd][:, 2], o[w][jd][:, 3]
            sel = T == 0  # warp 0, tig 0 lanes write (m, l)
            part_ml[row, split, G[sel], 0], part_ml[row, split, G[sel], 1] = m0[0][sel] * LN2, l0[0][sel]
            part_ml[row, split, G[sel] + 8, 0], part_ml[row, split, G[sel] + 8, 1] = m1[0][sel] * LN2, l1[0][sel]
    # mla_merge_kernel
    M = part_ml[..., 0].max(axis=1, keepdims=True)
    f = np.exp(part_ml[..., 0] - M)
    L = (part_ml[..., 1] * f).sum(axis=1)
    A = (part_acc * f[..., None]).sum(axis=1)
    return A / np.where(L > 0, L, 1.0)[..., None]


def reference_mla(q_lat, q_pe, cache, bt, row_seq, row_len, scale):
    out = np.zeros((q_lat.shape[0], H, K_LAT))
    for row in range(q_lat.shape[0]):
        seq, ln = int(row_seq[row]), int(row_len[row])
        toks = np.concatenate([cache[bt[seq, p]] for p in range((ln + K_PAGE - 1) // K_PAGE)])[:ln]  # [ln, 576]
        q = np.concatenate([q_lat[row], q_pe[row]], axis=1)  # [16, 576]
        s = q @ toks.T * scale
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[row] = p @ toks[:, :K_LAT]
    return out


@pytest.mark.parametrize("dtype,lens,splits", [("bf16", [37, 16], 2), ("fp16", [70, 5], 3), ("bf16", [129], 1),
                                               ("bf16", [20, 48, 9], 4)])
def test_mla_mma_kernel_emulation_matches_fp32_attention(dtype, lens, splits):
    rng = np.random.default_rng(len(lens) * 100 + splits)
    rows = len(lens)
    max_pages = max((ln + 15) // 16 for ln in lens)
    n_blocks = rows * max_pages + 3
    cache = round_to(rng.standard_normal((n_blocks, K_PAGE, K_ROW)), dtype)
    perm = rng.permutation(n_blocks)[: rows * max_pages]
    bt = perm.reshape(rows, max_pages).astype(np.int32)  # scattered pages
    q_lat = rng.standard_normal((rows, H, K_LAT)).astype(np.float32)
    q_pe = rng.standard_normal((rows, H, 64)).astype(np.float32)
    row_seq = np.arange(rows, dtype=np.int32)
    row_len = np.array(lens, dtype=np.int32)
    scale = 1.0 / np.sqrt(192.0)
    got = emulate_mla_mma(q_lat, q_pe, cache, bt, row_seq, row_len, splits, scale, dtype)
    want = reference_mla(q_lat.astype(np.float64), q_pe.astype(np.float64), cache, bt, row_seq, row_len, scale)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err < 2e-2, err
