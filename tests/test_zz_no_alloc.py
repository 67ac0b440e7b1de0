"""The allocation-free decode-attention entry point, called through its exported C symbol.

``barq_decode_attention_static`` takes its split-KV scratch from a static device array instead of
allocated memory; its results must match the allocating entry point (``ops.decode_attention``) on
consecutive calls that reuse the shared array.  This file sorts last so it also runs after every
other GPU test in one process.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
BS = 16
STATIC_BYTES = 8 * 1024 * 1024
E_SCRATCH = -101
E_ARGS = -103


def _lib():
    import barq_inference_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    f = lib.barq_decode_attention_static
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p] + \
        [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    need = lib.barq_decode_attention_static_need
    need.restype = ctypes.c_ulonglong
    need.argtypes = [ctypes.c_int] * 4
    err = lib.barq_static_strerror
    err.restype = ctypes.c_char_p
    err.argtypes = [ctypes.c_int]
    return f, need, err


def _case(Ls, H, Hkv, D, seed):
    g = torch.Generator().manual_seed(seed)
    nb = sum((L + BS - 1) // BS for L in Ls) + 4
    kc = torch.randn(nb, Hkv, BS, D, generator=g).half().to(DEV)
    vc = torch.randn(nb, Hkv, BS, D, generator=g).half().to(DEV)
    perm = torch.randperm(nb, generator=g).tolist()
    mb = max((L + BS - 1) // BS for L in Ls)
    bt = torch.zeros(len(Ls), mb, dtype=torch.int32)
    k = 0
    for i, L in enumerate(Ls):
        for j in range((L + BS - 1) // BS):
            bt[i, j] = perm[k]
            k += 1
    q = torch.randn(len(Ls), H, D, generator=g).bfloat16().to(DEV)
    lens = torch.tensor(Ls, dtype=torch.int32, device=DEV)
    return q, kc, vc, bt.to(DEV), lens


def _call_static(f, q, kc, vc, bt, lens, H, Hkv, D, scale, window, splits):
    B = q.shape[0]
    out = torch.empty(B, H * D, dtype=torch.float16, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    rc = f(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), 0, bt.data_ptr(), bt.shape[1], lens.data_ptr(), B, H, Hkv, D,
           BS, scale, window, splits, out.data_ptr(), 1, stream)
    return rc, out


def test_static_scratch_matches_allocating_entry_point():
    from barq_inference_b200 import ops

    f, need, err = _lib()
    cases = [  # two calls in a row with different shapes: the second reuses the array the first left behind
        ([1, 17, 300, 1024], 32, 8, 128, 0, 7),
        ([900, 33, 5], 8, 2, 64, 100, 3),
    ]
    for Ls, H, Hkv, D, window, splits in cases:
        q, kc, vc, bt, lens = _case(Ls, H, Hkv, D, seed=len(Ls))
        scale = 1 / math.sqrt(D)
        assert need(len(Ls), H, D, splits) <= STATIC_BYTES
        ref, _ = ops.decode_attention(q, kc, vc, bt, lens, H, Hkv, D, scale, window=window, splits=splits,
                                      want_q8=False, act_dtype=torch.float16)
        rc, out = _call_static(f, q, kc, vc, bt, lens, H, Hkv, D, scale, window, splits)
        torch.cuda.synchronize()
        assert rc == 0, err(rc).decode()
        assert torch.allclose(out.float(), ref.float(), atol=1e-2, rtol=1e-2), (out.float() - ref.float()).abs().max()


def test_static_scratch_rejects_oversized_shape():
    f, need, err = _lib()
    B, H, Hkv, D, splits = 64, 64, 8, 128, 64  # 4*(64*64*64*128 + ...) bytes > 8 MiB
    assert need(B, H, D, splits) > STATIC_BYTES
    q, kc, vc, bt, lens = _case([20] * B, H, Hkv, D, seed=5)
    rc, _ = _call_static(f, q, kc, vc, bt, lens, H, Hkv, D, 0.1, 0, splits)
    assert rc == E_SCRATCH
    assert b"static array" in err(rc)


def test_static_rejects_unsupported_group_size_before_launch():
    """H / Hkv = 16 is outside the kernels' {1, 2, 4, 8}: an argument error, nothing launched, and
    the thread's recorded CUDA error stays cudaSuccess."""
    import barq_inference_b200._C as C

    f, need, err = _lib()
    last = ctypes.CDLL(C.__file__).barq_static_last_cuda_error
    last.restype = ctypes.c_int
    q, kc, vc, bt, lens = _case([40, 7], 64, 4, 128, seed=9)
    rc, _ = _call_static(f, q, kc, vc, bt, lens, 64, 4, 128, 0.1, 0, 2)
    assert rc == E_ARGS
    assert b"{1, 2, 4, 8}" in err(rc)
    assert last() == 0
