"""tcgen05 prefill attention (``prefill_attention(..., impl=1)``, ``csrc/kernels/attn_prefill_tc.cu``)
against an fp32 torch reference and against the mma.sync kernel, then the tiny Llama runner on it.

Opt-in (``BARQ_TEST_PREFILL_TC=1``): the kernel is new and is checked on the CPU by emulating its
shared-memory layouts, descriptors and TMEM plan (``tests/test_tcgen05_emulation_cpu.py``) until a
B200 run of this file validates it; the model path keeps the mma.sync kernel by default
(``BARQ_PREFILL_TC=1`` selects the tcgen05 one)."""
import math
import os

import pytest
import torch

from barq_inference_b200 import ops

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("BARQ_TEST_PREFILL_TC") != "1",
                                 reason="opt-in: BARQ_TEST_PREFILL_TC=1 (kernel not yet validated on a GPU)")]
DEV = "cuda"


def _paged(Ls, Hkv, D, dtype, seed, nb_total=256):
    g = torch.Generator().manual_seed(seed)
    kc = torch.randn(nb_total, Hkv, 16, D, generator=g).to(dtype).to(DEV)
    vc = torch.randn(nb_total, Hkv, 16, D, generator=g).to(dtype).to(DEV)
    perm = torch.randperm(nb_total, generator=g).tolist()
    bt = torch.zeros(len(Ls), max((L + 15) // 16 for L in Ls), dtype=torch.int32)
    k = 0
    for i, L in enumerate(Ls):
        for j in range((L + 15) // 16):
            bt[i, j] = perm[k]
            k += 1
    return kc, vc, bt.to(DEV)


def _gather(cache, bt_row, L):
    blocks = [cache[int(b)] for b in bt_row[: (L + 15) // 16]]
    return torch.cat([b.transpose(0, 1) for b in blocks], 0)[:L].float().cpu()


@pytest.mark.parametrize("D,H,Hkv,cdt", [(128, 8, 2, torch.bfloat16), (64, 4, 2, torch.bfloat16),
                                          (128, 8, 2, torch.float16), (64, 4, 2, torch.float16)])
@pytest.mark.parametrize("window", [0, 100])
def test_prefill_tc_matches_fp32_and_mma_sync(D, H, Hkv, cdt, window):
    # (n_new, ctx): first chunk, later chunk, a one-token row, two full query tiles, a long prompt
    spec = [(70, 70), (130, 300), (1, 45), (256, 256), (600, 900)]
    Ls = [c for _, c in spec]
    kc, vc, bt = _paged(Ls, Hkv, D, cdt, seed=5)
    T = sum(n for n, _ in spec)
    q = torch.randn(T, H, D, device=DEV).bfloat16()
    qs = [0]
    for n, _ in spec:
        qs.append(qs[-1] + n)
    q_start = torch.tensor(qs, dtype=torch.int32, device=DEV)
    ctx = torch.tensor(Ls, dtype=torch.int32, device=DEV)
    scale = 1 / math.sqrt(D)
    max_q = max(n for n, _ in spec)
    ops.require_ext().gemm_clear_error()
    out = ops.prefill_attention(q, kc, vc, bt, q_start, ctx, max_q, H, Hkv, D, scale, window, impl=1)
    base = ops.prefill_attention(q, kc, vc, bt, q_start, ctx, max_q, H, Hkv, D, scale, window, impl=0)
    torch.cuda.synchronize()
    assert ops.gemm_error() == 0
    assert torch.isfinite(out.float()).all()
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
    assert (out.float() - base.float()).abs().max().item() < 2e-2


def test_tiny_runner_on_tcgen05_prefill(monkeypatch):
    """Tiny Llama: prefill logits with the tcgen05 kernel within 1e-2 of the fp32 reference."""
    from test_gpu_model import _run, _tiny
    from barq_inference_b200.models.reference import ReferenceModel
    from barq_inference_b200.models.runner import LlamaRunner

    monkeypatch.setenv("BARQ_PREFILL_TC", "1")
    cfg, tensors, prompt = _tiny()
    ref_logits = ReferenceModel(cfg, tensors).greedy(prompt, 1)[1]
    runner = LlamaRunner(cfg, tensors, DEV)
    runner.allocate_kv(64)
    lg = _run(runner, prompt, 0, list(range(1, 10)), decode=False)
    assert (lg - ref_logits[0]).abs().max().item() < 1e-2
