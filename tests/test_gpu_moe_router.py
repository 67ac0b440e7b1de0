"""MoE router-logits kernel (``ops.moe_router_logits``, ``moe_router_kernel`` in csrc/kernels/moe.cu)
against the f32 torch matmul, and the routed MoE layer with it.

Opt-in (``BARQ_TEST_MOE_ROUTER=1``): the kernel has not run on a GPU yet; the model path keeps the
library matmul unless ``BARQ_MOE_ROUTER=1``."""
import os

import pytest
import torch

from barq_inference_b200 import ops

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("BARQ_TEST_MOE_ROUTER") != "1",
                                 reason="opt-in: BARQ_TEST_MOE_ROUTER=1 (kernel not yet validated on a GPU)")]


@pytest.mark.parametrize("T,E,H,dt", [(1, 8, 4096, torch.bfloat16), (37, 64, 2048, torch.float16),
                                      (300, 160, 512, torch.bfloat16), (8, 256, 7168, torch.bfloat16)])
def test_router_logits_match_f32_matmul(T, E, H, dt):
    g = torch.Generator().manual_seed(T + E)
    x = torch.randn(T, H, generator=g).to(dt).cuda()
    w = (torch.randn(E, H, generator=g) / H ** 0.5).cuda()
    got = ops.moe_router_logits(x, w)
    ref = x.float() @ w.T
    torch.cuda.synchronize()
    assert (got - ref).abs().max().item() < 1e-4 * max(1.0, ref.abs().max().item())
    # strided rows (a view into a wider activation buffer)
    xw = torch.randn(T, H + 64, generator=g).to(dt).cuda()[:, :H]
    assert torch.allclose(ops.moe_router_logits(xw, w), xw.float() @ w.T, atol=1e-4, rtol=1e-4)


def test_moe_layer_routes_the_same_with_the_kernel(monkeypatch):
    from barq_inference_b200.models import POLICIES, preset, random_tensors
    from barq_inference_b200.models.reference import ReferenceModel
    from barq_inference_b200.models.runner import LlamaRunner
    from test_gpu_model import _run

    monkeypatch.setenv("BARQ_MOE_ROUTER", "1")
    cfg = preset("tiny-moe")
    tensors = random_tensors(cfg, POLICIES["tiny-moe"], seed=0)
    prompt = list(range(1, 40))
    ref_logits = ReferenceModel(cfg, tensors).greedy(prompt, 1)[1]
    runner = LlamaRunner(cfg, tensors, "cuda")
    runner.allocate_kv(64)
    lg = _run(runner, prompt, 0, list(range(1, 10)), decode=False)
    assert (lg - ref_logits[0]).abs().max().item() < 2e-2
