"""Sequence-parallel fused collectives (csrc/kernels/tp_fused.cu, the RS / AG modes of the tcgen05
GEMM) on one GPU, with W ranks emulated by W sets of buffers.

Each emulated rank's row-parallel GEMM pushes its output tiles into the owners' slots (EPI_RS_PUSH);
each owner's ``sp_reduce_norm_ag`` then adds the W partials into its residual rows, normalizes and
pushes the rows into every rank's gather buffer; finally a column-parallel GEMM waits on the gather
flags.  The launches run one after another on one stream, so every flag a kernel waits for was set
by an earlier kernel (no two kernels wait on each other).  Checked against a plain fp32 PyTorch
reference of the same layer: out = RMSNorm(x + sum_r X_r W_r^T) * w, then out @ V^T.
"""
import pytest
import torch

from barq_inference_b200 import ops
from barq_inference_b200.gguf import GGMLType, dequantize, quantize

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _qw(N, K, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * 0.02
    raw = quantize(w, GGMLType.Q4_K)
    return ops.QWeight.from_packed(raw, GGMLType.Q4_K, N, K, DEV), torch.from_numpy(
        dequantize(raw.numpy(), GGMLType.Q4_K, (N, K)))


def _i32(n):
    return torch.zeros(n, dtype=torch.int32, device=DEV)


@pytest.mark.parametrize("W", [1, 2, 3, 8])
@pytest.mark.parametrize("T", [37, 200])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_rs_reduce_norm_ag_gemm_matches_fp32(W, T, dt):
    C = ops.require_ext()
    H, Kr, N2 = 512, 256, 384  # hidden, per-rank K of the row-parallel GEMM, next GEMM's rows
    chunk = -(-T // W)
    max_tiles = -(-H // 128) * -(-T // 32)
    ws = [_qw(H, Kr, 10 + r) for r in range(W)]          # rank r's row-parallel shard
    xs = [torch.randn(T, Kr, generator=torch.Generator().manual_seed(20 + r)).to(dt) for r in range(W)]
    x0 = torch.randn(T, H, generator=torch.Generator().manual_seed(3))  # residual stream before the add
    nw = 1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(4))
    v, vref = _qw(N2, H, 30)

    # per-rank device state (every "peer" buffer is local memory here)
    slots = [torch.zeros(W * chunk * H, device=DEV) for _ in range(W)]
    rsf = [_i32(W * max_tiles) for _ in range(W)]
    ag = [torch.zeros(T, H, dtype=dt, device=DEV) for _ in range(W)]
    agf = [_i32(T) for _ in range(W)]
    epoch = [_i32(2) for _ in range(W)]
    done = [_i32(2) for _ in range(W)]
    site = 0
    for r in range(W):  # 1) row-parallel GEMMs, reduce-scatter fused into the epilogue
        w, _ = ws[r]
        C.qgemm_sp(*w.args(), xs[r].to(DEV), T, ops.EPI_RS_PUSH, None, None, None, H,
                   [s.data_ptr() for s in slots], [f.data_ptr() for f in rsf], epoch[r][site:site + 1], r, chunk,
                   max_tiles, None, None, 5.0)
    xloc = []
    for o in range(W):  # 2) owners: reduce + residual + RMSNorm + all-gather push
        a, b = min(T, o * chunk), min(T, o * chunk + chunk)
        xl = x0[a:b].clone().to(DEV)
        C.sp_reduce_norm_ag(xl, T, o, chunk, slots[o], rsf[o], W, max_tiles, C.gemm_tile_rows(T), -(-H // 128), None,
                            nw.to(DEV), 1e-5, [g.data_ptr() for g in ag], [f.data_ptr() for f in agf],
                            epoch[o][site:site + 1], done[o][site:site + 1], 5.0, int(dt == torch.float16), 0)
        xloc.append(xl)
    torch.cuda.synchronize()
    assert ops.gemm_error() == 0
    # fp32 reference
    part = sum(xs[r].float() @ ws[r][1].to(dt).float().T for r in range(W))
    xr = x0 + part
    normed = xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-5) * nw
    got_x = torch.cat([t.cpu() for t in xloc])
    assert torch.allclose(got_x, xr, atol=2e-3 * xr.abs().max().item(), rtol=1e-3), (got_x - xr).abs().max()
    for q in range(W):  # every rank's gather buffer holds every row
        assert torch.allclose(ag[q].float().cpu(), normed, atol=normed.abs().max().item() / 100, rtol=1e-2)
        assert int(agf[q].min()) == 1 and int(epoch[q][site]) == 1 and int(done[q][site]) == 0
    # 3) column-parallel GEMM consuming the gathered rows, waiting on their flags
    for q in range(W):
        y = torch.empty(T, N2, device=DEV)
        C.qgemm_sp(*v.args(), ag[q], T, ops.EPI_STORE_F32, y, None, None, N2, [], [], None, q, 0, 0,
                   agf[q], epoch[q][site:site + 1], 5.0)
        y_ref = ag[q].float().cpu() @ vref.to(dt).float().T
        assert ops.gemm_error() == 0
        assert torch.allclose(y.cpu(), y_ref, atol=2e-3 * y_ref.abs().max().item(), rtol=1e-2)


def test_ag_wait_times_out_on_missing_rows():
    """A gather flag that nothing sets: the GEMM's bounded wait gives up, records 0x400 in the error
    word and the context stays usable."""
    C = ops.require_ext()
    v, _ = _qw(128, 256, 1)
    x = torch.zeros(70, 256, dtype=torch.float16, device=DEV)
    flags, ep = _i32(70), torch.ones(1, dtype=torch.int32, device=DEV)
    y = torch.empty(70, 128, device=DEV)
    C.qgemm_sp(*v.args(), x, 70, ops.EPI_STORE_F32, y, None, None, 128, [], [], None, 0, 0, 0, flags, ep, 0.05)
    torch.cuda.synchronize()
    assert ops.gemm_error() & 0xF00 == 0x400
    ops.require_ext().gemm_clear_error()
    assert ops.gemm_error() == 0
    torch.zeros(1, device=DEV).add_(1)  # the context still runs work
    torch.cuda.synchronize()


def test_expert_parallel_all_to_all_world_of_one_matches_fused_moe():
    """The expert-parallel dispatch / grouped GEMMs / combine (moe.cu ep_* kernels) as a world of one
    rank holding every expert, against the single-GPU fused MoE block on the same rows."""
    from barq_inference_b200.models import POLICIES, preset, random_tensors
    from barq_inference_b200.models.moe import MoEBlock

    C = ops.require_ext()
    cfg = preset("tiny-moe")
    tensors = random_tensors(cfg, POLICIES["tiny-moe"], seed=2)
    moe = MoEBlock(cfg, tensors, "blk.0.", DEV)
    rows, H, E, k = 37, cfg.hidden, moe.E, moe.k
    g = torch.Generator().manual_seed(8)
    hb = torch.randn(rows, H, generator=g).half().to(DEV)
    x0 = torch.randn(rows, H, generator=g).to(DEV)

    class _R:  # what MoEBlock.forward reads from its runner
        ser_threshold, fused_moe, x2 = 0.0, True, True

    ref = x0.clone()
    moe.forward(_R(), None, hb, rows, ref)
    i32 = lambda n: torch.zeros(n, dtype=torch.int32, device=DEV)  # noqa: E731
    cap = rows * k
    cnt, cf, df, yf = i32(E), i32(1), i32(1), i32(1)
    rx = torch.zeros(cap, H, dtype=torch.float16, device=DEV)
    ys = torch.zeros(cap, H, device=DEV)
    counts, cursor, off, pos = i32(E), i32(E), i32(E + 1), i32(rows * k * 2)
    ids, wts = i32(rows * k).view(rows, k), torch.zeros(rows, k, device=DEV)
    epoch, done, d = i32(1), i32(2), i32(cap + E)
    for call in range(2):  # two layers' worth: the epoch and the zeroed counters carry over
        logits = hb.float() @ moe.router.T
        ra = moe._route_args(0.0)
        C.moe_route(logits.contiguous(), k, int(ra["sigmoid"]), int(ra["renorm"]), ra["n_group"], ra["topk_group"],
                    0.0, ra["scale"], hb, ids, wts, counts, d, d, d, d.float(), d, None)
        args = (0, E, E, k, rows, ids, wts, counts, cursor, [cnt.data_ptr()], [cf.data_ptr()], hb, [rx.data_ptr()],
                [df.data_ptr()], pos, off, [ys.data_ptr()], [yf.data_ptr()])
        C.ep_call(0, *args, None, epoch, done, cap, 5.0)
        h = ops.gemm_grouped(moe.gate_up, rx, off, E, ops.EPI_SWIGLU_Q8)
        ops.gemm_grouped(moe.down, h, off, E, ops.EPI_STORE_F32, out=ys)
        out = x0.clone()
        C.ep_call(1, *args, out, epoch, done, cap, 5.0)
        torch.cuda.synchronize()
        assert ops.gemm_error() == 0
        assert int(epoch) == call + 1 and int(counts.abs().sum()) == 0 and int(cursor.abs().sum()) == 0
        assert int(off[-1]) == int((wts > 0).sum())
        assert torch.allclose(out, ref, atol=2e-3 * ref.abs().max().item(), rtol=1e-3), (out - ref).abs().max()
