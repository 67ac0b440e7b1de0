"""End-to-end engine checks on the GPU against the fp32 reference forward (tiny config)."""
import pytest
import torch

from barq_inference_b200.engine.engine import Engine, EngineConfig
from barq_inference_b200.engine.sampling_params import SamplingParams
from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.models.reference import ReferenceModel
from barq_inference_b200.models.runner import LlamaRunner, StepInput

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tiny():
    cfg = preset("tiny")
    tensors = random_tensors(cfg, POLICIES["tiny"], seed=0)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab, (64,), generator=g).tolist()
    return cfg, tensors, prompt


def _run(runner, toks, start, table, decode):
    T = len(toks)
    pos = list(range(start, start + T))
    slots = [table[p // 16] * 16 + p % 16 for p in pos]
    d = lambda a, dt: torch.tensor(a, dtype=dt, device=DEV)  # noqa: E731
    bt = d([table], torch.int32)
    inp = StepInput(d(toks, torch.int32), d(pos, torch.int32), d(slots, torch.int64), bt,
                    d([start + T], torch.int32), d([T - 1], torch.int64), decode,
                    q_start=d([0, T], torch.int32), max_q=T)
    return runner.forward(inp)[0].float().cpu()


def test_tiny_logits_match_reference():
    """Tiny config check: logits within 1e-2 of the fp32 dequantized reference."""
    cfg, tensors, prompt = _tiny()
    ref = ReferenceModel(cfg, tensors)
    ref_tokens, ref_logits = ref.greedy(prompt, 64)
    runner = LlamaRunner(cfg, tensors, DEV)
    runner.allocate_kv(64)
    table = list(range(1, 10))
    lg = _run(runner, prompt, 0, table, decode=False)
    err = (lg - ref_logits[0]).abs().max().item()
    assert err < 1e-2, err
    # teacher-forced decode over the reference's greedy continuation
    pos = len(prompt)
    worst = err
    for i, t in enumerate(ref_tokens[:-1]):
        lg = _run(runner, [t], pos, table, decode=True)
        pos += 1
        worst = max(worst, (lg - ref_logits[i + 1]).abs().max().item())
    assert worst < 1e-2, worst


def test_engine_generate_greedy_graph_vs_eager():
    cfg, tensors, prompt = _tiny()
    outs = []
    for graphs in (False, True):
        eng = Engine(cfg, tensors, EngineConfig(max_num_seqs=8, max_model_len=512, num_blocks=256,
                                                cuda_graphs=graphs))
        prompts = [prompt, prompt[:17], prompt[5:50]]
        res = eng.generate(prompts, SamplingParams.greedy_params(max_tokens=16))
        outs.append([r.tokens for r in res])
        assert all(len(r.tokens) == 16 for r in res)
    assert outs[0] == outs[1]


def test_engine_chunked_prefill_matches_whole():
    cfg, tensors, prompt = _tiny()
    res = []
    for budget in (8192, 24):
        eng = Engine(cfg, tensors, EngineConfig(max_num_seqs=4, max_model_len=512, num_blocks=128,
                                                max_num_batched_tokens=budget, cuda_graphs=False))
        res.append(eng.generate([prompt], SamplingParams.greedy_params(max_tokens=8))[0].tokens)
    assert res[0] == res[1]


def test_engine_sampling_runs():
    cfg, tensors, prompt = _tiny()
    eng = Engine(cfg, tensors, EngineConfig(max_num_seqs=4, max_model_len=512, num_blocks=128))
    r = eng.generate([prompt] * 3, SamplingParams(max_tokens=12, temperature=0.9, top_k=40, top_p=0.95, seed=3))
    assert all(len(x.tokens) == 12 for x in r)
    assert all(0 <= t < cfg.vocab for x in r for t in x.tokens)


def test_small_q4k_gemm_and_gemv_paths_match_reference():
    """Llama-3-style (Q4_K + Q6_K head) small model: prefill on the tcgen05 GEMM path and decode on the
    GEMV path both track the fp32 reference."""
    cfg = preset("llama3-8b", n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024, vocab=1000,
                 max_ctx=512)
    tensors = random_tensors(cfg, POLICIES["llama3-8b"], seed=4)
    g = torch.Generator().manual_seed(2)
    prompt = torch.randint(0, cfg.vocab, (100,), generator=g).tolist()
    ref = ReferenceModel(cfg, tensors)
    ref_tokens, ref_logits = ref.greedy(prompt, 4)
    runner = LlamaRunner(cfg, tensors, DEV)
    runner.allocate_kv(64)
    table = list(range(1, 12))
    lg = _run(runner, prompt, 0, table, decode=False)
    scale = ref_logits[0].abs().max().item()
    assert (lg - ref_logits[0]).abs().max().item() < 2e-2 * scale
    pos = len(prompt)
    for i, t in enumerate(ref_tokens[:-1]):
        lg = _run(runner, [t], pos, table, decode=True)
        pos += 1
        assert (lg - ref_logits[i + 1]).abs().max().item() < 1e-2 * scale


def test_batched_decode_gemm_path_matches_gemv_path():
    cfg = preset("llama3-8b", n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024, vocab=1000,
                 max_ctx=512)
    tensors = random_tensors(cfg, POLICIES["llama3-8b"], seed=4)
    prompts = [list(range(i, i + 20 + i)) for i in range(20)]
    outs = []
    for gemm in (True, False):
        eng = Engine(cfg, tensors, EngineConfig(max_num_seqs=32, max_model_len=256, num_blocks=256, cuda_graphs=False))
        eng.runner.use_gemm = gemm
        outs.append([r.tokens for r in eng.generate(prompts, SamplingParams.greedy_params(max_tokens=6))])
    same = sum(a == b for a, b in zip(outs[0], outs[1]))
    assert same >= 14, same  # bf16 GEMM vs two-term int8 GEMV: random-init logits are near-ties


def test_dense_prefill_path_matches_fused(monkeypatch):
    """Large-T prefill route (dequantize the weight once + dense GEMM) == fused-dequant GEMM route."""
    import barq_inference_b200.models.runner as rmod

    cfg, tensors, prompt = _tiny()
    outs = []
    for dense_t in (0, 16):
        monkeypatch.setattr(rmod, "DENSE_T", dense_t)
        runner = LlamaRunner(cfg, tensors, DEV)
        runner.allocate_kv(64)
        outs.append(_run(runner, prompt, 0, list(range(1, 10)), decode=False))
    assert (outs[0] - outs[1]).abs().max().item() < 2e-2


def test_fp8_kv_cache_logits_close_to_fp16():
    """fp8 (e4m3) KV cache: prefill + teacher-forced decode logits stay close to the fp16-cache run,
    and the engine's graph and eager paths agree token for token."""
    cfg, tensors, prompt = _tiny()
    table = list(range(1, 10))
    logits = {}
    for dt in (torch.float16, torch.float8_e4m3fn):
        runner = LlamaRunner(cfg, tensors, DEV, kv_dtype=dt)
        runner.allocate_kv(64)
        out = [_run(runner, prompt, 0, table, decode=False)]
        for i, t in enumerate(prompt[:16]):
            out.append(_run(runner, [t], len(prompt) + i, table, decode=True))
        logits[dt] = torch.stack(out)
    a, b = logits[torch.float16], logits[torch.float8_e4m3fn]
    rel = ((a - b).norm(dim=-1) / a.norm(dim=-1)).max().item()
    assert rel < 0.1, rel
    outs = []
    for graphs in (False, True):
        eng = Engine(cfg, tensors, EngineConfig(max_num_seqs=4, max_model_len=512, num_blocks=128,
                                                cuda_graphs=graphs, kv_dtype="fp8"))
        outs.append([r.tokens for r in eng.generate([prompt, prompt[:20]],
                                                    SamplingParams.greedy_params(max_tokens=12))])
    assert outs[0] == outs[1]


def test_multimodal_prompt_embeds_on_gpu():
    """Image-patch embeddings replace placeholder rows on the device path (whole and chunked
    prefill), matching the fp32 reference forward given the same embeddings."""
    from barq_inference_b200.models.vision import ImageInput, LlavaModel

    cfg, tensors, prompt = _tiny()
    img = ImageInput.solid_rgb(224, 224, [10, 200, 30])
    toks = []
    for budget in (8192, 40):
        eng = Engine(cfg, tensors, EngineConfig(max_num_seqs=4, max_model_len=512, num_blocks=128,
                                                max_num_batched_tokens=budget, cuda_graphs=False))
        vlm = LlavaModel(eng)
        toks.append(vlm.generate(prompt[:8], img, SamplingParams.greedy_params(max_tokens=4)).tokens)
    assert toks[0] == toks[1]
    e = vlm.image_embeddings(img).cpu()
    ref = ReferenceModel(cfg, tensors)
    lg = ref.forward(prompt[:8] + [0] * e.shape[0], {}, embeds=(8, e))[-1]
    assert toks[0][0] == int(lg.argmax())


def test_long_context_32k_yarn_prefill_vs_decode():
    """A 32k-token context (YaRN x4 over an 8k original window): the last token's logits from the
    decode path (split-KV decode attention over 2048 pages) match the prefill path's (paged prefill
    attention) for the same position."""
    import dataclasses

    cfg = dataclasses.replace(preset("tiny", max_ctx=32768), rope_scaling="yarn", rope_factor=4.0,
                              rope_orig_ctx=8192)
    tensors = random_tensors(cfg, POLICIES["tiny"], seed=0)
    L = 32768 - 8
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, cfg.vocab, (L,), generator=g).tolist()
    runner = LlamaRunner(cfg, tensors, DEV)
    runner.allocate_kv(L // 16 + 8)
    table = list(range(1, L // 16 + 2))
    for s in range(0, L - 1, 4096):
        _run(runner, prompt[s:min(s + 4096, L - 1)], s, table, decode=False)
    dec = _run(runner, [prompt[L - 1]], L - 1, table, decode=True)
    pre = _run(runner, prompt[L - 4096:], L - 4096, table, decode=False)  # recompute the last chunk
    assert torch.isfinite(dec).all()
    rel = ((dec - pre).norm() / pre.norm()).item()
    assert rel < 2e-2, rel
    assert int(dec.argmax()) == int(pre.argmax())


def test_speculative_greedy_matches_plain_greedy():
    """Draft + target (one batched verify forward per round): greedy output is token-for-token the
    target's plain greedy output, whatever the draft; a draft identical to the target is always
    accepted."""
    from barq_inference_b200.engine.speculative import SpeculativeConfig, SpeculativeDecoder

    cfg, tensors, prompt = _tiny()
    ec = lambda: EngineConfig(max_num_seqs=4, max_model_len=512, num_blocks=128, cuda_graphs=False)  # noqa: E731
    target = Engine(cfg, tensors, ec())
    plain = target.generate([prompt[:24]], SamplingParams.greedy_params(max_tokens=20))[0].tokens
    other = Engine(cfg, random_tensors(cfg, POLICIES["tiny"], seed=7), ec())
    out = SpeculativeDecoder(target, other, SpeculativeConfig(4)).generate(
        prompt[:24], SamplingParams.greedy_params(max_tokens=20))
    assert out.tokens == plain
    same = SpeculativeDecoder(target, Engine(cfg, tensors, ec()), SpeculativeConfig(4, adaptive=False)).generate(
        prompt[:24], SamplingParams.greedy_params(max_tokens=20))
    assert same.tokens == plain and same.acceptance_rate > 0.99
    sampled = SpeculativeDecoder(target, other, SpeculativeConfig(3)).generate(
        prompt[:24], SamplingParams(temperature=0.8, top_k=40, max_tokens=16, seed=5, ignore_eos=True))
    assert len(sampled.tokens) == 16 and all(0 <= t < cfg.vocab for t in sampled.tokens)


def test_sliding_window_decode_matches_reference_and_skips_dead_pages():
    """A 40-token sliding window on the device kernels, teacher-forced (greedy token equality is not
    used: random-init logits have near-ties that any rounding difference flips): (1) prefill and
    decode logits track the fp32 reference with the same window within 1e-2; (2) a block table
    whose pages behind the window point at a dummy page full of garbage gives the same logits as
    the intact table (pages outside the window are never used); (3) the engine frees those pages
    while generating and returns every page at the end."""
    import dataclasses

    cfg0, tensors, prompt = _tiny()
    cfg = dataclasses.replace(cfg0, sliding_window=40)
    ref = ReferenceModel(cfg, tensors)
    ref_tokens, ref_logits = ref.greedy(prompt, 24)
    runner = LlamaRunner(cfg, tensors, DEV)
    runner.allocate_kv(64)
    for K, V in runner.kv:  # page 0 is the dummy page: garbage that must never be attended to
        K[0].fill_(1000.0)
        V[0].fill_(1000.0)
    table = list(range(1, 12))
    lg = _run(runner, prompt, 0, table, decode=False)
    assert (lg - ref_logits[0]).abs().max().item() < 1e-2
    pos = len(prompt)
    for i, t in enumerate(ref_tokens[:-1]):
        dead = max(0, pos - 40 + 1) // 16
        trimmed = [0] * dead + table[dead:]
        a = _run(runner, [t], pos, table, decode=True)
        b = _run(runner, [t], pos, trimmed, decode=True)
        assert (a - ref_logits[i + 1]).abs().max().item() < 1e-2, i
        assert (a - b).abs().max().item() < 1e-4, i
        pos += 1
    eng = Engine(cfg, tensors, EngineConfig(max_num_seqs=4, max_model_len=512, num_blocks=64,
                                            max_num_batched_tokens=32))
    out = eng.generate([prompt], SamplingParams.greedy_params(max_tokens=48))[0].tokens
    assert len(out) == 48 and eng.sched.n_window_freed >= 3
    assert eng.blocks.n_used == 1  # only the engine's own dummy page is still held


def test_fp8_kv_row_scales_keep_values_beyond_e4m3_range():
    """K/V rows with magnitudes in the thousands (e4m3 saturates at 448): the per-row scales of the
    fp8 cache keep decode and prefill attention within a few percent of the fp16-cache result."""
    from barq_inference_b200 import ops
    from barq_inference_b200.models.rope import rope_cos_sin

    cfg = preset("tiny")
    H, Hkv, D, T = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, 40
    g = torch.Generator().manual_seed(3)
    qkv = (torch.randn(T, (H + 2 * Hkv) * D, generator=g) * 1000).to(DEV)
    cos, sin = rope_cos_sin(cfg, 512, DEV)
    pos = torch.arange(T, dtype=torch.int32, device=DEV)
    slots = (torch.arange(T, device=DEV) + 16).long()  # pages 1..3
    bt = torch.tensor([[1, 2, 3, 0]], dtype=torch.int32, device=DEV)
    outs = {}
    for dt in (torch.float16, torch.float8_e4m3fn):
        kc = torch.zeros(5, Hkv, 16, D, device=DEV).to(dt)
        vc = torch.zeros(5, Hkv, 16, D, device=DEV).to(dt)
        sc = (torch.ones(5, Hkv, 16, device=DEV), torch.ones(5, Hkv, 16, device=DEV)) if dt != torch.float16 else None
        q = ops.rope_kv_write(qkv, pos, slots, cos, sin, H, Hkv, D, cfg.rot_dim, cfg.rope_neox, kc, vc, kv_scales=sc)
        q = (q.float() / 1000).bfloat16()  # keep the scores in a sane range; K/V stay large
        lens = torch.tensor([T], dtype=torch.int32, device=DEV)
        dec, _ = ops.decode_attention(q[-1:].contiguous(), kc, vc, bt, lens, H, Hkv, D, D ** -0.5, want_q8=False,
                                      act_dtype=torch.float16, kv_scales=sc)
        pre = ops.prefill_attention(q, kc, vc, bt, torch.tensor([0, T], dtype=torch.int32, device=DEV), lens, T,
                                    H, Hkv, D, D ** -0.5, act_dtype=torch.float16, kv_scales=sc)
        outs[dt] = (dec.float().cpu(), pre.float().cpu())
    for a, b in zip(outs[torch.float16], outs[torch.float8_e4m3fn]):
        rel = ((a - b).norm() / a.norm()).item()
        assert rel < 0.06, rel
