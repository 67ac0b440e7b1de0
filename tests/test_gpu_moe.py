"""MoE block on the GPU (routing kernels + grouped tcgen05 GEMMs) against the fp32 reference."""
import pytest
import torch

from barq_inference_b200 import ops
from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.models.reference import ReferenceModel, moe_route
from barq_inference_b200.models.runner import LlamaRunner, StepInput

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(runner, toks, start, table, decode):
    T = len(toks)
    pos = list(range(start, start + T))
    slots = [table[p // 16] * 16 + p % 16 for p in pos]
    d = lambda a, dt: torch.tensor(a, dtype=dt, device=DEV)  # noqa: E731
    inp = StepInput(d(toks, torch.int32), d(pos, torch.int32), d(slots, torch.int64), d([table], torch.int32),
                    d([start + T], torch.int32), d([T - 1], torch.int64), decode,
                    q_start=d([0, T], torch.int32), max_q=T)
    return runner.forward(inp)[0].float().cpu()


@pytest.mark.parametrize("E,k,ser", [(8, 2, 0.0), (64, 6, 0.0), (8, 2, 0.3)])
def test_route_kernel_matches_reference(E, k, ser):
    T, H = 40, 128
    g = torch.Generator().manual_seed(E + k)
    logits = torch.randn(T, E, generator=g)
    x = torch.randn(T, H, generator=g).half()
    cfg = preset("tiny-moe", n_experts=E, n_experts_used=k)
    r = ops.MoeRouting(T, E, k, H, torch.float16, DEV)
    ops.moe_route(logits.to(DEV), x.to(DEV), k, r, ser_threshold=ser)
    ids_ref, w_ref = moe_route(logits, cfg, ser)
    ids, w = r.ids.cpu(), r.weights.cpu()
    assert torch.equal(ids.long(), ids_ref)
    assert torch.allclose(w, w_ref, atol=1e-5)
    off = r.off.cpu()
    kept = (w_ref > 0)
    for e in range(E):
        assert off[e + 1] - off[e] == int(((ids_ref == e) & kept).sum())
    n = int(off[E])
    xs, tok, rw = r.xs[:n].cpu(), r.row_tok[:n].cpu(), r.row_w[:n].cpu()
    assert torch.equal(xs, x[tok.long()])
    for row in range(n):
        t = int(tok[row])
        e = int(torch.searchsorted(off[1:], torch.tensor(row), right=True))
        j = int((ids_ref[t] == e).nonzero()[0, 0])
        assert abs(float(rw[row]) - float(w_ref[t, j])) < 1e-6
    assert int(r.counts.sum()) == 0  # left zero for the next call


@pytest.mark.parametrize("fused", [True, False])
def test_tiny_moe_logits_match_reference(fused):
    cfg = preset("tiny-moe")
    tensors = random_tensors(cfg, POLICIES["tiny-moe"], seed=3)
    ref = ReferenceModel(cfg, tensors)
    g = torch.Generator().manual_seed(7)
    prompt = torch.randint(0, cfg.vocab, (24,), generator=g).tolist()
    ref_tokens, ref_logits = ref.greedy(prompt, 6)
    runner = LlamaRunner(cfg, tensors, DEV)
    runner.fused_moe = fused
    runner.allocate_kv(32)
    table = list(range(1, 8))
    lg = _run(runner, prompt, 0, table, decode=False)
    worst = (lg - ref_logits[0]).abs().max().item()
    pos = len(prompt)
    for i, t in enumerate(ref_tokens[:-1]):
        lg = _run(runner, [t], pos, table, decode=True)
        pos += 1
        worst = max(worst, (lg - ref_logits[i + 1]).abs().max().item())
    assert worst < 2e-2, worst


def test_tiny_deepseek_mla_logits_match_reference():
    """DeepSeek-V2 runner (latent cache, absorbed MLA kernel, dense + MoE with a shared expert)."""
    from barq_inference_b200.models.deepseek2 import DeepseekV2Runner

    cfg = preset("tiny-ds")
    tensors = random_tensors(cfg, POLICIES["tiny-ds"], seed=5)
    ref = ReferenceModel(cfg, tensors)
    g = torch.Generator().manual_seed(9)
    prompt = torch.randint(0, cfg.vocab, (40,), generator=g).tolist()
    ref_tokens, ref_logits = ref.greedy(prompt, 5)
    runner = DeepseekV2Runner(cfg, tensors, DEV)
    runner.allocate_kv(32)
    table = list(range(1, 10))
    lg = _run(runner, prompt, 0, table, decode=False)
    worst = (lg - ref_logits[0]).abs().max().item()
    pos = len(prompt)
    for i, t in enumerate(ref_tokens[:-1]):
        lg = _run(runner, [t], pos, table, decode=True)
        pos += 1
        worst = max(worst, (lg - ref_logits[i + 1]).abs().max().item())
    assert worst < 3e-2, worst


@pytest.mark.parametrize("name", ["tiny-moe", "tiny-ds"])
def test_engine_moe_families_graph_vs_eager(name):
    """Engine end to end on the MoE / MLA families: CUDA-graph decode == eager decode."""
    from barq_inference_b200.engine.engine import Engine, EngineConfig
    from barq_inference_b200.engine.sampling_params import SamplingParams

    cfg = preset(name)
    tensors = random_tensors(cfg, POLICIES[name], seed=11)
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, cfg.vocab, (30,), generator=g).tolist()
    outs = []
    for graphs in (False, True):
        eng = Engine(cfg, tensors, EngineConfig(max_num_seqs=4, max_model_len=256, num_blocks=64, cuda_graphs=graphs))
        res = eng.generate([prompt, prompt[:9]], SamplingParams.greedy_params(max_tokens=8))
        outs.append([r.tokens for r in res])
        assert all(len(r.tokens) == 8 for r in res)
    assert outs[0] == outs[1]
