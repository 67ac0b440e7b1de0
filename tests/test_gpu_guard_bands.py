"""Guard bands around kernel outputs, and the device-side index checks.

Each output is a view into a larger buffer whose margins hold a sentinel; after the kernel the
margins must be untouched (no kernel writes outside its output).  Ids outside the table and
block-table entries outside the cache are recorded in the device error word and never
dereferenced (the checks use indices just past the end, so even an unchecked read would stay
inside the allocation)."""
import pytest
import torch

from barq_inference_b200 import ops
from barq_inference_b200.gguf import GGMLType, quantize

pytestmark = pytest.mark.gpu
DEV = "cuda"
G = 4096  # guard elements on each side
SENT = -4096.0  # exact in fp16, bf16 and f32


def _guarded(n, dtype=torch.float32):
    full = torch.full((n + 2 * G,), SENT, dtype=dtype, device=DEV)
    return full, full[G:G + n]


def _intact(full):
    f = full.float()
    return bool((f[:G] == SENT).all()) and bool((f[-G:] == SENT).all())


def _qw(N, K, t=GGMLType.Q4_K, seed=0):
    w = torch.randn(N, K, generator=torch.Generator().manual_seed(seed)) * 0.02
    return ops.QWeight.from_packed(quantize(w, t), t, N, K, DEV)


@pytest.mark.parametrize("T", [1, 5, 37, 300])
def test_gemm_and_gemv_outputs_stay_inside(T):
    N, K = 384, 1024
    w = _qw(N, K)
    x = torch.randn(T, K, device=DEV).half()
    for mode in (ops.EPI_STORE_F32, ops.EPI_ADD_F32):
        for ks in (1, 0):
            full, v = _guarded(T * N)
            v.zero_()
            ops.gemm(w, x, mode, out=v.view(T, N), k_splits=ks)
            torch.cuda.synchronize()
            assert _intact(full), (mode, ks)
    gu = ops.interleave_gate_up(_qw(256, K, seed=1), _qw(256, K, seed=2))
    full, v = _guarded(T * 256, torch.float16)
    ops.gemm(gu, x, ops.EPI_SWIGLU_Q8, out=v.view(T, 256))
    torch.cuda.synchronize()
    assert _intact(full)
    if T <= 8:
        xa = ops.quantize_q8(torch.randn(T, K, device=DEV), True)
        full, v = _guarded(T * N)
        ops.gemv(w, xa, T, ops.EPI_STORE_F32, out=v.view(T, N), x2=True)
        torch.cuda.synchronize()
        assert _intact(full)


def test_embedding_out_of_range_id_is_recorded_not_read():
    C = ops.require_ext()
    C.gemm_clear_error()
    V, H = 64, 256
    w = _qw(V, H, GGMLType.Q8_0)
    full, v = _guarded(3 * H)
    C.embed_gather(*w.args(), torch.tensor([1, V, 2], dtype=torch.int32, device=DEV), v.view(3, H))
    torch.cuda.synchronize()
    assert _intact(full)
    assert ops.gemm_error() == 0xB00
    assert float(v.view(3, H)[1].abs().sum()) == 0.0 and float(v.view(3, H)[0].abs().sum()) > 0
    C.gemm_clear_error()


def test_decode_attention_bad_block_table_entry_is_recorded():
    C = ops.require_ext()
    C.gemm_clear_error()
    nb, Hkv, D, H = 6, 2, 64, 4
    kc = torch.randn(nb, Hkv, 16, D, device=DEV).half()
    vc = torch.randn(nb, Hkv, 16, D, device=DEV).half()
    bt = torch.tensor([[1, nb]], dtype=torch.int32, device=DEV)  # second page is past the cache
    lens = torch.tensor([30], dtype=torch.int32, device=DEV)
    q = torch.randn(1, H, D, device=DEV).bfloat16()
    out, _ = ops.decode_attention(q, kc, vc, bt, lens, H, Hkv, D, 0.125, want_q8=False)
    torch.cuda.synchronize()
    assert ops.gemm_error() == 0xA00
    assert torch.isfinite(out.float()).all()
    C.gemm_clear_error()
