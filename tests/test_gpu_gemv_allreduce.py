"""Fused streaming GEMV + tensor-parallel all-reduce (EPI_AR_PUSH) on one GPU.

The multi-rank protocol is exercised in one process by giving the kernel a "world of 2" whose
second rank is emulated with local buffers: either its slot in our receive buffer already holds
this call's (epoch, value) words (the exchange completes, x gains W a + that partial, and our
tile words reach the emulated peer's buffer), or nothing ever arrives (the bounded wait runs out,
the error word is set, x is unchanged, the context stays usable).  The real 2-GPU path is covered
by test_gpu_tp.py."""
import pytest
import torch

from barq_inference_b200 import ops
from barq_inference_b200.gguf import GGMLType, dequantize, quantize

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _setup(t, N, K, B, world, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * 0.02
    raw = quantize(w, t)
    qw = ops.QWeight.from_packed(raw, t, N, K, DEV)
    ref = torch.from_numpy(dequantize(raw.numpy(), t, (N, K)))
    x = torch.randn(B, K, device=DEV)
    xa = ops.quantize_q8(x, True)
    y_ref = ops.gemv(qw, xa, B, ops.EPI_STORE_F32).cpu()  # the plain streaming GEMV
    bufs = [torch.zeros(2, world, B * N, dtype=torch.int64, device=DEV) for _ in range(world)]  # [j][slot][B*N]
    epoch = torch.zeros(2, dtype=torch.int32, device=DEV)
    done = torch.zeros(2, dtype=torch.int32, device=DEV)
    return qw, ref, xa, y_ref, bufs, epoch, done


def _push(bufs, epoch, done, rank, wait_s, skip=0):
    tabs = [torch.tensor([b[j].data_ptr() for b in bufs], dtype=torch.int64, device=DEV) for j in (0, 1)]

    def args(j, T, H):
        return tabs[j], epoch, done, rank, wait_s, skip
    return args


def _words(vals: torch.Tensor, ep: int) -> torch.Tensor:
    """f32 values -> (epoch << 32 | bits) 64-bit words."""
    bits = vals.float().contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return bits | (ep << 32)


def _unwords(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    return (w & 0xFFFFFFFF).to(torch.int32).view(torch.float32), w >> 32


@pytest.mark.parametrize("t,B", [(GGMLType.Q4_K, 1), (GGMLType.Q6_K, 2), (GGMLType.Q8_0, 5)])
def test_gemv_allreduce_world1(t, B):
    N, K = 512, 1024
    qw, _, xa, y_ref, bufs, epoch, done = _setup(t, N, K, B, 1)
    res = torch.randn(B, N, device=DEV)
    x = res.clone()
    for j, it in ((0, 1), (1, 1), (0, 2)):
        ops.gemv_allreduce(qw, xa, B, x, _push(bufs, epoch, done, 0, 5.0), j)
        torch.cuda.synchronize()
        assert int(epoch[j]) == it and int(done.abs().sum()) == 0
    assert ops.gemm_error() == 0
    assert torch.allclose(x.cpu(), res.cpu() + 3 * y_ref, atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("t", [GGMLType.Q4_K, GGMLType.Q4_0])
def test_gemv_allreduce_emulated_peer(t):
    N, K, B = 384, 512, 2
    qw, _, xa, y_ref, bufs, epoch, done = _setup(t, N, K, B, 2, seed=1)
    peer_partial = torch.randn(B * N, device=DEV)
    bufs[0][1, 1] = _words(peer_partial, 1)   # rank 1's words (epoch 1) in our receive buffer j=1
    res = torch.randn(B, N, device=DEV)
    x = res.clone()
    ops.gemv_allreduce(qw, xa, B, x, _push(bufs, epoch, done, 0, 5.0), 1)
    torch.cuda.synchronize()
    assert ops.gemm_error() == 0
    want = res.cpu() + y_ref + peer_partial.view(B, N).cpu()
    assert torch.allclose(x.cpu(), want, atol=1e-3, rtol=1e-4)
    # our tile words (epoch 1) reached the emulated peer's buffer, slot 0
    vals, eps = _unwords(bufs[1][1, 0])
    assert torch.allclose(vals.view(B, N).cpu(), y_ref, atol=1e-5) and bool((eps == 1).all())
    assert int(epoch[1]) == 1 and int(done[1]) == 0


def test_gemv_allreduce_peer_timeout_is_reported():
    C = ops.require_ext()
    C.gemm_clear_error()
    N, K, B = 256, 512, 1
    qw, _, xa, _, bufs, epoch, done = _setup(GGMLType.Q4_K, N, K, B, 2, seed=2)
    x = torch.randn(B, N, device=DEV)
    before = x.clone()
    ops.gemv_allreduce(qw, xa, B, x, _push(bufs, epoch, done, 0, 0.3), 0)
    torch.cuda.synchronize()
    err = C.gemm_error()
    assert err & 0xF00 == 0x300 and err & 0xFF == 1, hex(err)
    assert torch.equal(x, before)            # nothing added without the peer
    assert int(epoch[0]) == 1 and int(done[0]) == 0  # still advanced / reset: ranks stay aligned
    C.gemm_clear_error()
    assert float((torch.ones(8, device=DEV) * 2).sum()) == 16.0  # the context is still usable
