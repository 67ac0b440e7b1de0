"""Tensor-core MLA decode kernel (``mla_attention(..., impl=1)``) against an fp32 torch reference of
absorbed MLA attention and against the CUDA-core kernel, then the tiny DeepSeek runner on it.

Opt-in (``BARQ_TEST_MLA_MMA=1``): the kernel is new and is checked on the CPU by lane-level
emulation (``tests/test_mla_mma_emulation_cpu.py``) until a B200 run of this file validates it; the
model path keeps the CUDA-core kernel by default (``BARQ_MLA_MMA`` selects the tensor-core one)."""
import os

import pytest
import torch

from barq_inference_b200 import ops

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("BARQ_TEST_MLA_MMA") != "1",
                                 reason="opt-in: BARQ_TEST_MLA_MMA=1 (kernel not yet validated on a GPU)")]
DEV = "cuda"


def _case(lens, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    rows, H, qdim = len(lens), 16, 192
    pages = max((n + 15) // 16 for n in lens)
    nb = rows * pages + 2
    cache = torch.randn(nb, 16, 576, generator=g).to(dtype).to(DEV)
    bt = (torch.randperm(nb - 1, generator=g)[: rows * pages] + 1).view(rows, pages).to(torch.int32).to(DEV)
    q_lat = torch.randn(rows, H, 512, generator=g).to(DEV)
    q = torch.randn(rows, H * qdim, generator=g).to(DEV)
    rs = torch.arange(rows, dtype=torch.int32, device=DEV)
    rl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    return cache, bt, q_lat, q, rs, rl


def _reference(cache, bt, q_lat, q, rl, scale, rope_off=128, qdim=192):
    out = []
    for r in range(q_lat.shape[0]):
        n = int(rl[r])
        toks = cache[bt[r, : (n + 15) // 16].long()].reshape(-1, 576)[:n].float()
        qpe = q[r].view(16, qdim)[:, rope_off:rope_off + 64]
        qq = torch.cat([q_lat[r], qpe], 1)
        p = torch.softmax(qq @ toks.T * scale, -1)
        out.append(p @ toks[:, :512])
    return torch.stack(out)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("lens,splits", [([37, 16], 2), ([1, 300, 64], 3), ([4096] * 4, 16), ([129], 1),
                                         ([20, 48, 9, 1000], 5)])
def test_mla_mma_kernel_matches_reference(dtype, lens, splits):
    cache, bt, q_lat, q, rs, rl = _case(lens, dtype, seed=len(lens) + splits)
    scale = 192 ** -0.5
    want = _reference(cache, bt, q_lat, q, rl, scale)
    got = ops.mla_attention(q_lat, q, 192, 128, cache, bt, rs, rl, 16, splits, scale, impl=1)
    old = ops.mla_attention(q_lat, q, 192, 128, cache, bt, rs, rl, 16, splits, scale, impl=0)
    torch.cuda.synchronize()
    err = ((got - want).abs().max() / want.abs().max()).item()
    assert err < 2e-2, err
    assert ((got - old).abs().max() / old.abs().max()).item() < 2e-2


def test_tiny_deepseek_runner_on_the_tensor_core_kernel(monkeypatch):
    monkeypatch.setenv("BARQ_MLA_MMA", "1")
    from test_gpu_moe import test_tiny_deepseek_mla_logits_match_reference

    test_tiny_deepseek_mla_logits_match_reference()
