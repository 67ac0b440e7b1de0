"""Decode is deterministic: the same step run twice gives bit-identical logits.

Every cross-CTA sum on the decode path (stream-K pieces of the streaming GEMV, split-K tiles of the
tcgen05 GEMM, the MoE combine, split-KV attention) is added in a fixed order, never with
floating-point atomics, so rounding does not depend on which CTA finishes first.  Checked at batch 1
(streaming GEMV path) and batch 64 (tcgen05 GEMM path), eagerly and through a captured CUDA graph,
on the tiny config and on two Llama-3-8B-shaped layers (Q4_K, Q6_K head).
"""
import dataclasses

import pytest
import torch

from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.models.runner import LlamaRunner, StepInput

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(B, ctx, pages_per_seq, vocab, seed):
    g = torch.Generator().manual_seed(seed)
    toks = torch.randint(0, vocab, (B,), generator=g)
    tables = torch.arange(1, 1 + B * pages_per_seq, dtype=torch.int32).reshape(B, pages_per_seq)
    pos = torch.full((B,), ctx, dtype=torch.int32)
    slots = tables[:, ctx // 16].long() * 16 + ctx % 16
    d = lambda a, dt: a.to(DEV, dt)  # noqa: E731
    return StepInput(d(toks, torch.int32), d(pos, torch.int32), d(slots, torch.int64), d(tables, torch.int32),
                     d(pos + 1, torch.int32), torch.arange(B, device=DEV), True)


def _prefill(runner, B, ctx, pages_per_seq, vocab):
    """Fill every sequence's first ``ctx`` positions with one batched prefill."""
    g = torch.Generator().manual_seed(7)
    toks = torch.randint(0, vocab, (B * ctx,), generator=g)
    tables = torch.arange(1, 1 + B * pages_per_seq, dtype=torch.int32).reshape(B, pages_per_seq)
    pos = torch.arange(ctx, dtype=torch.int32).repeat(B)
    seq = torch.arange(B).repeat_interleave(ctx)
    slots = tables[seq, pos.long() // 16].long() * 16 + pos.long() % 16
    d = lambda a, dt: a.to(DEV, dt)  # noqa: E731
    inp = StepInput(d(toks, torch.int32), d(pos, torch.int32), d(slots, torch.int64), d(tables, torch.int32),
                    torch.full((B,), ctx, dtype=torch.int32, device=DEV),
                    (torch.arange(B, device=DEV) + 1) * ctx - 1, False,
                    q_start=torch.arange(B + 1, dtype=torch.int32, device=DEV) * ctx, max_q=ctx)
    runner.forward(inp)


def _check(cfg, policy, B, ctx):
    tensors = random_tensors(cfg, policy, seed=0, device=DEV)
    runner = LlamaRunner(cfg, tensors, DEV)
    pages = (ctx + 1 + 15) // 16
    runner.allocate_kv(1 + B * pages)
    _prefill(runner, B, ctx, pages, cfg.vocab)
    inp = _inputs(B, ctx, pages, cfg.vocab, seed=3)
    a = runner.forward(inp)[0].float().clone()
    b = runner.forward(inp)[0].float().clone()
    assert torch.isfinite(a).all()
    assert torch.equal(a, b), (a - b).abs().max().item()
    # the same step replayed from a captured CUDA graph
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        runner.forward(inp)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = runner.forward(inp)[0]
    graph.replay()
    c = out.float().clone()
    graph.replay()
    d = out.float().clone()
    assert torch.equal(c, d), (c - d).abs().max().item()
    assert torch.equal(a, c), (a - c).abs().max().item()


@pytest.mark.parametrize("B", [1, 64])
def test_tiny_decode_bit_identical(B):
    _check(preset("tiny"), POLICIES["tiny"], B, ctx=40)


@pytest.mark.parametrize("B", [1, 64])
def test_llama8b_layers_decode_bit_identical(B):
    cfg = dataclasses.replace(preset("llama3-8b"), n_layers=2)
    _check(cfg, POLICIES["llama3-8b"], B, ctx=100)


def test_moe_decode_bit_identical():
    cfg = preset("tiny-moe")
    _check(cfg, POLICIES["tiny-moe"], 64, ctx=24)
