"""Numerics of the sm_100a kernels against plain PyTorch fp32 references of the same op."""
import math

import numpy as np
import pytest
import torch

from barq_inference_b200 import ops
from barq_inference_b200.gguf import GGMLType, dequantize, quantize
from barq_inference_b200.models.rope import apply_rope_ref

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _qw(t, N, K, seed=0, std=0.02):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * std
    raw = quantize(w, t)
    qw = ops.QWeight.from_packed(raw, t, N, K, DEV)
    ref = torch.from_numpy(dequantize(raw.numpy(), t, (N, K)))
    return qw, ref, raw


def _q8_deq(a: ops.Q8Act) -> torch.Tensor:
    q = a.q.float().cpu()
    d = a.s[..., 0].cpu()
    out = (q.view(q.shape[0], -1, 32) * d[..., None]).reshape(q.shape)
    if a.x2:
        ql = a.ql.float().cpu()
        dl = a.dl[..., 0].cpu()
        out = out + (ql.view(q.shape[0], -1, 32) * dl[..., None]).reshape(q.shape)
    return out


TYPES = [GGMLType.Q4_0, GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q5_K, GGMLType.Q6_K, GGMLType.IQ4_NL]


@pytest.mark.parametrize("t", TYPES)
def test_planar_roundtrip(t):
    qw, _, raw = _qw(t, 64, 512)
    assert torch.equal(qw.to_gguf_rows().cpu(), raw)


@pytest.mark.parametrize("t", TYPES)
def test_dequant_rows_exact(t):
    qw, ref, _ = _qw(t, 48, 512)
    out = ops.dequant_rows(qw).float().cpu()
    assert torch.allclose(out, ref.bfloat16().float(), atol=0, rtol=0)


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("B", [1, 3, 8])
@pytest.mark.parametrize("x2", [False, True])
def test_gemv(t, B, x2):
    N, K = 264, 1024
    qw, ref, _ = _qw(t, N, K)
    x = torch.randn(B, K, device=DEV)
    xa = ops.quantize_q8(x, x2)
    xd = _q8_deq(xa)
    # q8 quantization itself
    bound = x.abs().max().cpu() / 127 * 0.51 * (1 / 120 if x2 else 1)
    assert (xd - x.cpu()).abs().max() <= bound + 1e-6
    y = ops.gemv(qw, xa, B, ops.EPI_STORE_F32).cpu()
    y_ref = xd @ ref.T
    assert torch.allclose(y, y_ref, atol=2e-4, rtol=2e-3), (y - y_ref).abs().max()
    # residual-add epilogue
    base = torch.randn(B, N, device=DEV)
    out = base.clone()
    ops.gemv(qw, xa, B, ops.EPI_ADD_F32, out=out)
    assert torch.allclose(out.cpu(), base.cpu() + y_ref, atol=2e-4, rtol=2e-3)


@pytest.mark.parametrize("t", [GGMLType.Q4_K, GGMLType.Q4_0])
@pytest.mark.parametrize("x2", [False, True])
def test_gemv_swiglu_epilogue(t, x2):
    F, K, B = 128, 512, 4
    g, gref, _ = _qw(t, F, K, seed=1)
    u, uref, _ = _qw(t, F, K, seed=2)
    w = ops.interleave_gate_up(g, u)
    x = torch.randn(B, K, device=DEV)
    xa = ops.quantize_q8(x, x2)
    xd = _q8_deq(xa)
    h = ops.gemv(w, xa, B, ops.EPI_SWIGLU_Q8, x2=x2)
    gg, uu = xd @ gref.T, xd @ uref.T
    h_ref = torch.nn.functional.silu(gg) * uu
    hd = _q8_deq(h)
    assert torch.allclose(hd, h_ref, atol=h_ref.abs().max() / 100, rtol=2e-2)


@pytest.mark.parametrize("t", [GGMLType.Q4_K, GGMLType.Q6_K, GGMLType.Q8_0])
@pytest.mark.parametrize("B", [1, 2])
@pytest.mark.parametrize("x2", [False, True])
def test_gemv_fused_norm(t, B, x2):
    """RMSNorm inside the streaming GEMV vs the fp32 reference of rmsnorm(h) @ W^T, with the same
    tolerance as the unfused GEMV (the two paths may round a few activation codes differently)."""
    N, K = 384, 2048
    qw, ref, _ = _qw(t, N, K, seed=4)
    h = torch.randn(B, K, device=DEV) * 3
    nw = torch.rand(K, device=DEV) + 0.5
    hn = (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-5) * nw).cpu()
    y_ref = hn @ ref.T
    tol = y_ref.abs().max() * (2e-3 if x2 else 2e-2)
    y = ops.gemv(qw, None, B, ops.EPI_STORE_F32, x2=x2, norm=(h, nw, 1e-5)).cpu()
    assert (y - y_ref).abs().max() <= tol, (y - y_ref).abs().max()
    _, hq = ops.rmsnorm(h.clone(), nw, 1e-5, want_q8=True, x2=x2)
    y_unfused = ops.gemv(qw, hq, B, ops.EPI_STORE_F32, x2=x2).cpu()
    assert (y_unfused - y_ref).abs().max() <= tol
    if t == GGMLType.Q4_K:
        g2, ref2, _ = _qw(t, N, K, seed=5)
        w = ops.interleave_gate_up(qw, g2)
        hs = _q8_deq(ops.gemv(w, None, B, ops.EPI_SWIGLU_Q8, x2=x2, norm=(h, nw, 1e-5)))
        hs_ref = torch.nn.functional.silu(hn @ ref.T) * (hn @ ref2.T)
        assert (hs - hs_ref).abs().max() <= hs_ref.abs().max() / 50


@pytest.mark.parametrize("t", TYPES)
def test_dequant_dense_matches_oracle(t):
    N, K = 300, 512
    qw, ref, _ = _qw(t, N, K, seed=6)
    for dt in (torch.float16, torch.bfloat16):
        d = ops.dequant_dense(qw, dtype=dt).float().cpu()
        # the GEMM's operand numerics: per-block scale and min rounded to the operand type, one FMA
        tol = ref.abs().max() * (2e-3 if dt == torch.float16 else 1.6e-2)
        assert (d - ref).abs().max() <= tol, (t, dt, (d - ref).abs().max())


def test_bf16_gemv():
    N, K, B = 100, 688, 3
    w = torch.randn(N, K) * 0.02
    qw = ops.QWeight.from_packed(quantize(w, GGMLType.F16), GGMLType.F16, N, K, DEV)
    x = torch.randn(B, K, device=DEV).bfloat16()
    y = ops.gemv(qw, None, B, ops.EPI_STORE_F32, xb=x).cpu()
    y_ref = x.float().cpu() @ w.half().float().bfloat16().float().T
    assert torch.allclose(y, y_ref, atol=1e-3, rtol=1e-2)


def test_rmsnorm_fused_add():
    T, H = 5, 4096
    x = torch.randn(T, H, device=DEV)
    a = torch.randn(T, H, device=DEV)
    w = torch.rand(H, device=DEV) + 0.5
    x0 = x.clone()
    ob, oq = ops.rmsnorm(x, w, 1e-5, add=a, want_bf16=True, want_q8=True, x2=True)
    s = x0 + a
    ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-5) * w
    assert torch.allclose(x, s, atol=1e-6)
    assert torch.allclose(ob.float(), ref, atol=2e-2, rtol=1e-2)
    assert torch.allclose(_q8_deq(oq), ref.cpu(), atol=ref.abs().max().item() / 5000)


@pytest.mark.parametrize("neox,cdt", [(False, torch.float16), (True, torch.float16), (True, torch.float8_e4m3fn)])
def test_rope_kv_write(neox, cdt):
    from barq_inference_b200.models.config import preset
    from barq_inference_b200.models.rope import rope_cos_sin

    cfg = preset("tiny", max_ctx=256)
    H, Hkv, D, T = 4, 2, 64, 7
    cos, sin = rope_cos_sin(cfg, 256, DEV)
    qkv = torch.randn(T, (H + 2 * Hkv) * D, device=DEV)
    pos = torch.tensor([3, 17, 40, 41, 100, 200, 255], dtype=torch.int32, device=DEV)
    nb = 32
    kc = torch.zeros(nb, Hkv, 16, D, dtype=cdt, device=DEV)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([5, 16 * 3 + 2, 16 * 7 + 15, 1, 16 * 9, 16 * 31 + 4, 16 * 2 + 8], dtype=torch.int64,
                         device=DEV)
    q = ops.rope_kv_write(qkv, pos, slots, cos, sin, H, Hkv, D, D, neox, kc, vc)
    x = qkv.view(T, H + 2 * Hkv, D)
    c, s = cos[pos.long()].cpu(), sin[pos.long()].cpu()
    q_ref = apply_rope_ref(x[:, :H].cpu(), c, s, neox)
    k_ref = apply_rope_ref(x[:, H:H + Hkv].cpu(), c, s, neox)
    assert torch.allclose(q.float().cpu(), q_ref, atol=2e-2, rtol=1e-2)
    # fp8 e4m3: 3 mantissa bits, so a stored value is within 1/16 relative of the exact one
    tol = dict(atol=3e-3, rtol=1e-3) if cdt == torch.float16 else dict(atol=2e-3, rtol=0.07)
    for t in range(T):
        blk, off = int(slots[t]) // 16, int(slots[t]) % 16
        assert torch.allclose(kc[blk, :, off].float().cpu(), k_ref[t], **tol)
        assert torch.allclose(vc[blk, :, off].float().cpu(), x[t, H + Hkv:].cpu(), **tol)


def _paged(Ls, Hkv, D, nb_total=256, dtype=torch.float16, seed=0):
    g = torch.Generator().manual_seed(seed)
    kc = (torch.randn(nb_total, Hkv, 16, D, generator=g)).to(dtype).to(DEV)
    vc = (torch.randn(nb_total, Hkv, 16, D, generator=g)).to(dtype).to(DEV)
    perm = torch.randperm(nb_total, generator=g).tolist()
    mb = max((L + 15) // 16 for L in Ls)
    bt = torch.zeros(len(Ls), mb, dtype=torch.int32)
    k = 0
    for i, L in enumerate(Ls):
        for j in range((L + 15) // 16):
            bt[i, j] = perm[k]
            k += 1
    return kc, vc, bt.to(DEV)


def _gather(cache, bt_row, L):
    blocks = [cache[int(b)] for b in bt_row[: (L + 15) // 16]]
    return torch.cat([b.transpose(0, 1) for b in blocks], 0)[:L].float().cpu()  # [L, Hkv, D]


@pytest.mark.parametrize("D,H,Hkv,cdt", [(128, 32, 8, torch.float16), (64, 4, 2, torch.float16),
                                          (128, 8, 8, torch.float16), (128, 32, 8, torch.float8_e4m3fn),
                                          (64, 4, 2, torch.float8_e4m3fn), (128, 32, 8, torch.bfloat16)])
@pytest.mark.parametrize("window", [0, 40])
def test_decode_attention(D, H, Hkv, cdt, window):
    Ls = [1, 17, 300, 1024]
    kc, vc, bt = _paged(Ls, Hkv, D, dtype=cdt)
    B = len(Ls)
    q = torch.randn(B, H, D, device=DEV).bfloat16()
    lens = torch.tensor(Ls, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(D)
    out, oq = ops.decode_attention(q, kc, vc, bt, lens, H, Hkv, D, scale, window=window)
    G = H // Hkv
    for b, L in enumerate(Ls):
        k = _gather(kc, bt[b].cpu(), L).repeat_interleave(G, 1)
        v = _gather(vc, bt[b].cpu(), L).repeat_interleave(G, 1)
        s = torch.einsum("hd,lhd->hl", q[b].float().cpu(), k) * scale
        if window:
            s[:, : max(0, L - window)] = -float("inf")
        o = torch.einsum("hl,lhd->hd", torch.softmax(s, -1), v).reshape(-1)
        assert torch.allclose(out[b].float().cpu(), o, atol=1e-2, rtol=1e-2), (b, (out[b].float().cpu() - o).abs().max())
        assert torch.allclose(_q8_deq(oq)[b], o, atol=o.abs().max() / 60)


@pytest.mark.parametrize("D,H,Hkv,cdt", [(128, 8, 2, torch.bfloat16), (64, 4, 2, torch.bfloat16),
                                          (128, 8, 2, torch.float8_e4m3fn), (64, 4, 2, torch.float16)])
@pytest.mark.parametrize("window", [0, 100])
def test_prefill_attention(D, H, Hkv, cdt, window):
    # (n_new, ctx): first chunk, a later chunk of a long prompt, a one-token row
    spec = [(70, 70), (130, 300), (1, 45), (256, 256)]
    Ls = [c for _, c in spec]
    kc, vc, bt = _paged(Ls, Hkv, D, seed=3, dtype=cdt)
    T = sum(n for n, _ in spec)
    q = torch.randn(T, H, D, device=DEV).bfloat16()
    qs = [0]
    for n, _ in spec:
        qs.append(qs[-1] + n)
    q_start = torch.tensor(qs, dtype=torch.int32, device=DEV)
    ctx = torch.tensor(Ls, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(D)
    out = ops.prefill_attention(q, kc, vc, bt, q_start, ctx, max(n for n, _ in spec), H, Hkv, D, scale, window)
    G = H // Hkv
    for i, (n, L) in enumerate(spec):
        k = _gather(kc, bt[i].cpu(), L).repeat_interleave(G, 1)
        v = _gather(vc, bt[i].cpu(), L).repeat_interleave(G, 1)
        qq = q[qs[i]:qs[i + 1]].float().cpu()
        s = torch.einsum("thd,lhd->htl", qq, k) * scale
        qpos = torch.arange(L - n, L)[:, None]
        kpos = torch.arange(L)[None]
        m = kpos > qpos
        if window:
            m |= kpos <= qpos - window
        s = s.masked_fill(m[None], -float("inf"))
        o = torch.einsum("htl,lhd->thd", torch.softmax(s, -1), v).reshape(n, -1)
        got = out[qs[i]:qs[i + 1]].float().cpu()
        assert torch.allclose(got, o, atol=2e-2, rtol=2e-2), (i, (got - o).abs().max())


@pytest.mark.parametrize("t", [GGMLType.Q8_0, GGMLType.Q4_K, GGMLType.Q6_K])
def test_embed_gather(t):
    qw, ref, _ = _qw(t, 100, 512)
    ids = torch.tensor([0, 5, 99, 5, 42], dtype=torch.int32, device=DEV)
    out = ops.embed(qw, ids).cpu()
    assert torch.allclose(out, ref[ids.long().cpu()], atol=1e-6)


def _sample(logits, temp, k=0, p=1.0, minp=0.0, seed=1, step=0):
    B = logits.shape[0]
    f = lambda v, dt: torch.full((B,), v, dtype=dt, device=DEV)  # noqa: E731
    ids, lp = ops.sample(logits.clone(), f(temp, torch.float32), f(k, torch.int32), f(p, torch.float32),
                         f(minp, torch.float32), f(seed, torch.int64), f(step, torch.int32), want_logprob=True)
    return ids.cpu(), lp.cpu()


def test_sampler_greedy():
    logits = torch.randn(6, 128256, device=DEV)
    ids, _ = _sample(logits, 0.0)
    assert torch.equal(ids.long(), logits.argmax(-1).cpu())


def test_sampler_topk_topp_distribution():
    V = 1000
    base = torch.randn(V) * 2
    logits = base.to(DEV).repeat(4000, 1)
    ids, lp = _sample(logits, 1.0, k=10)
    top10 = set(torch.topk(base, 10).indices.tolist())
    assert set(ids.tolist()) <= top10
    probs = torch.softmax(base[list(top10)], 0)
    counts = torch.bincount(ids.long(), minlength=V)[list(top10)].float() / ids.numel()
    assert (counts - probs).abs().max() < 0.04
    # nucleus without top-k (Gumbel path)
    ids2, _ = _sample(logits, 1.0, p=0.5)
    sp, si = torch.sort(torch.softmax(base, 0), descending=True)
    keep = set(si[: int((sp.cumsum(0) < 0.5).sum()) + 1].tolist())
    assert set(ids2.tolist()) <= keep
    # deterministic for a fixed seed/step
    ids3, _ = _sample(logits[:8], 1.0, k=10, seed=7, step=3)
    ids4, _ = _sample(logits[:8], 1.0, k=10, seed=7, step=3)
    assert torch.equal(ids3, ids4)


def test_sampler_penalties_and_mask():
    V = 64
    logits = torch.zeros(1, V, device=DEV)
    logits[0, 5] = 3.0
    logits[0, 9] = 2.9
    hist = torch.tensor([[5, 5, -1]], dtype=torch.int32, device=DEV)
    pen = torch.tensor([[1.0, 0.1, 0.0]], device=DEV)
    f = lambda v, dt: torch.full((1,), v, dtype=dt, device=DEV)  # noqa: E731
    ids, _ = ops.sample(logits.clone(), f(0.0, torch.float32), f(0, torch.int32), f(1.0, torch.float32),
                        f(0.0, torch.float32), f(0, torch.int64), f(0, torch.int32), penalties=pen, history=hist)
    assert int(ids) == 9  # 3.0 - 2*0.1 < 2.9
    mask = torch.zeros(1, 2, dtype=torch.int32, device=DEV)
    mask[0, 0] = 1 << 3
    ids, _ = ops.sample(logits.clone(), f(0.0, torch.float32), f(0, torch.int32), f(1.0, torch.float32),
                        f(0.0, torch.float32), f(0, torch.int64), f(0, torch.int32), allow_mask=mask)
    assert int(ids) == 3


GEMM_TYPES = [GGMLType.Q4_K, GGMLType.Q6_K, GGMLType.Q5_K, GGMLType.Q8_0, GGMLType.Q4_0, GGMLType.IQ4_NL]


@pytest.mark.parametrize("t", GEMM_TYPES)
@pytest.mark.parametrize("T", [1, 16, 32, 37, 64, 200, 300])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gemm_tc(t, T, dt):
    N, K = 384, 1024
    qw, ref, _ = _qw(t, N, K, seed=5)
    x = torch.randn(T, K, device=DEV).to(dt)
    y_ref = x.float().cpu() @ ref.to(dt).float().T
    tol = y_ref.abs().max().item() * 2e-3
    for ks in (1, 0):
        y = ops.gemm(qw, x, ops.EPI_STORE_F32, k_splits=ks).cpu()
        assert ops.gemm_error() == 0
        assert torch.allclose(y, y_ref, atol=tol, rtol=1e-2), (ks, (y - y_ref).abs().max())
    base = torch.randn(T, N, device=DEV)
    out = base.clone()
    ops.gemm(qw, x, ops.EPI_ADD_F32, out=out)
    assert torch.allclose(out.cpu(), base.cpu() + y_ref, atol=tol, rtol=1e-2)
    yb = ops.gemm(qw, x, ops.EPI_STORE_BF16)
    assert yb.dtype == dt
    assert torch.allclose(yb.float().cpu(), y_ref, atol=tol + y_ref.abs().max().item() / 128, rtol=1e-2)


@pytest.mark.parametrize("T", [5, 130])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gemm_tc_swiglu_and_ragged_n(T, dt):
    F, K = 192, 512
    g, gref, _ = _qw(GGMLType.Q4_K, F, K, seed=1)
    u, uref, _ = _qw(GGMLType.Q4_K, F, K, seed=2)
    w = ops.interleave_gate_up(g, u)
    x = torch.randn(T, K, device=DEV).to(dt)
    h = ops.gemm(w, x, ops.EPI_SWIGLU_Q8).float().cpu()
    xf = x.float().cpu()
    h_ref = torch.nn.functional.silu(xf @ gref.to(dt).float().T) * (xf @ uref.to(dt).float().T)
    assert torch.allclose(h, h_ref, atol=h_ref.abs().max().item() / 60, rtol=2e-2)
    # N not a multiple of the 128-row tile
    qw, ref, _ = _qw(GGMLType.Q4_K, 200, K, seed=3)
    y = ops.gemm(qw, x).cpu()
    y_ref = xf @ ref.to(dt).float().T
    assert torch.allclose(y, y_ref, atol=y_ref.abs().max().item() * 2e-3, rtol=1e-2)


def test_spec_verify_kernel_preserves_target_distribution():
    """K14 on the device: the first emitted token of the rejection step follows the target
    distribution p_0 whatever the draft proposed (the speculative-sampling guarantee); greedy
    accepts exactly the prefix that matches the target's argmax."""
    C = ops.require_ext()
    g = torch.Generator().manual_seed(4)
    V, k = 12, 3
    ps = torch.softmax(torch.randn(k + 1, V, generator=g) * 2, -1).to(DEV)
    qs = torch.softmax(torch.randn(k, V, generator=g) * 2, -1).to(DEV)
    out = torch.empty(k + 2, dtype=torch.int32, device=DEV)
    counts = torch.zeros(V)
    n = 6000
    dg = torch.Generator().manual_seed(9)
    for step in range(n):
        d = torch.multinomial(qs.cpu(), 1, generator=dg)[:, 0]  # drafts sampled from q
        C.spec_verify(ps, qs, d.to(DEV), 0, 77, step, out)
        r = out.cpu()
        assert 0 <= int(r[0]) <= k
        counts[int(r[1])] += 1
    emp = counts / n
    assert (emp - ps[0].cpu()).abs().max().item() < 0.025, (emp, ps[0])
    # greedy: drafts = target argmax for the first two positions, then a mismatch
    tgt = ps.argmax(-1).cpu()
    d = tgt[:k].clone()
    d[2] = (d[2] + 1) % V
    C.spec_verify(ps, None, d.to(DEV), 1, 0, 0, out)
    r = out.cpu().tolist()
    assert r[0] == 2 and r[1:4] == [int(tgt[0]), int(tgt[1]), int(tgt[2])]


def test_sampler_topk_ties_and_short_rows():
    """Top-k selection on a 128256-token row: of 40 tokens tied at the top, exactly k = 20 stay in
    play (ties go to the lower index), and a row with fewer than k tokens within 80 of the max
    samples among those only."""
    V = 128256
    g = torch.Generator().manual_seed(2)
    lg = torch.randn(V, generator=g)
    lg[100:140] = 9.0  # 40 tokens tied at the top, k = 20
    ids, _ = _sample(lg.to(DEV).repeat(2000, 1), 1.0, k=20)
    assert set(ids.tolist()) == set(range(100, 120))
    short = torch.full((V,), -1000.0)
    short[[7, 70000, 128000]] = torch.tensor([1.0, 0.5, 0.0])
    ids, _ = _sample(short.to(DEV).repeat(1000, 1), 1.0, k=50)
    assert set(ids.tolist()) <= {7, 70000, 128000} and len(set(ids.tolist())) == 3
