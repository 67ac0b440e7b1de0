"""KV session export / import: CPU engine end to end, and the GPU engine's paged gather/scatter and
prefix-cache donation on CPU tensors."""
import types

import pytest
import torch

from barq_inference_b200.engine.cpu_engine import CPUEngine
from barq_inference_b200.engine.kv_cache import BlockManager
from barq_inference_b200.engine.prefix_cache import RadixPrefixCache
from barq_inference_b200.engine.sampling_params import SamplingParams
from barq_inference_b200.engine.session import export_session, import_session, load_session
from barq_inference_b200.models import POLICIES, preset, random_tensors


def test_cpu_session_roundtrip(tmp_path):
    cfg = preset("tiny", n_layers=2, vocab=500, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=0)
    system = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(1)).tolist()
    path = str(tmp_path / "s.pt")
    export_session(CPUEngine(cfg, t, max_model_len=256), system, path)
    prompt = system + [5, 6, 7]
    p = SamplingParams.greedy_params(max_tokens=5)
    want = CPUEngine(cfg, t, max_model_len=256).generate([prompt], p)[0].tokens
    eng = CPUEngine(cfg, t, max_model_len=256)
    assert import_session(eng, path) == 40
    got = eng.generate([prompt], p)[0].tokens
    assert got == want
    assert eng.timings["prefill_tokens"] == 3  # only the new suffix was prefilled
    again = eng.generate([system], p)[0].tokens  # the exact session prompt: only its last token runs
    assert again == CPUEngine(cfg, t, max_model_len=256).generate([system], p)[0].tokens
    assert eng.timings["prefill_tokens"] == 4
    other = preset("tiny", n_layers=1, vocab=500, max_ctx=256)
    with pytest.raises(ValueError):
        import_session(CPUEngine(other, random_tensors(other, POLICIES["tiny"], seed=0)), path)


def _stub(nb=32, bs=16, L=2, H=2, D=8, dtype=torch.float16):
    cfg = types.SimpleNamespace(arch="llama", n_layers=L, n_kv_heads=H, head_dim=D, is_mla=False)
    blocks = BlockManager(nb, bs)
    kv = [(torch.zeros(nb, H, bs, D, dtype=dtype), torch.zeros(nb, H, bs, D, dtype=dtype)) for _ in range(L)]
    return types.SimpleNamespace(cfg=cfg, runner=types.SimpleNamespace(kv=kv), blocks=blocks,
                                 prefix_cache=RadixPrefixCache(blocks), ecfg=types.SimpleNamespace(tp=1, pp=1))


def test_paged_session_gather_scatter(tmp_path):
    a = _stub()
    toks = list(range(100, 140))  # 2 full pages + 8 tokens
    tbl = a.blocks.allocate(3)
    g = torch.Generator().manual_seed(0)
    for K, V in a.runner.kv:
        K.copy_(torch.randn(K.shape, generator=g).half())
        V.copy_(torch.randn(V.shape, generator=g).half())
    a.prefix_cache.insert(toks, tbl)
    path = str(tmp_path / "p.pt")
    st = export_session(a, toks + [1], path)
    st = load_session(path)
    assert st["tokens"].tolist() == toks[:32] and st["kv"]["k.0"].shape == (32, 2, 8)
    # row p of the export is position p: page p // 16, slot p % 16
    K0 = a.runner.kv[0][0]
    assert torch.equal(st["kv"]["k.0"][17], K0[tbl[1], :, 1])
    b = _stub()
    used0 = b.blocks.n_used
    assert import_session(b, st) == 32
    blocks, n = b.prefix_cache.match(toks + [1])
    assert n == 32 and b.blocks.n_used == used0 + 2  # held by the prefix cache only
    for (Ka, Va), (Kb, Vb) in zip(a.runner.kv, b.runner.kv):
        assert torch.equal(Ka[tbl[:2]], Kb[blocks]) and torch.equal(Va[tbl[:2]], Vb[blocks])
    c = _stub()
    c.prefix_cache = None
    with pytest.raises(ValueError):
        import_session(c, st)


def test_paged_session_fp8_pages():
    a = _stub(dtype=torch.float8_e4m3fn)
    toks = list(range(16))
    tbl = a.blocks.allocate(1)
    for K, V in a.runner.kv:
        K.copy_(torch.randn(K.shape).to(torch.float8_e4m3fn))
    a.prefix_cache.insert(toks, tbl)
    st = export_session(a, toks + [0])
    b = _stub(dtype=torch.float16)  # fp8 rows imported into an fp16 cache
    assert import_session(b, st) == 16
    blocks, _ = b.prefix_cache.match(toks + [0])
    assert torch.equal(b.runner.kv[1][0][blocks[0]], a.runner.kv[1][0][tbl[0]].to(torch.float16))


def test_cli_prompt_cache(tmp_path, caplog):
    """``run --prompt-cache``: the first run writes the session, the second reuses it (CPU engine)."""
    import logging

    from barq_inference_b200.cli import main

    path = str(tmp_path / "m.gguf")
    pc = str(tmp_path / "p.session")
    assert main(["make-random-gguf", "--arch", "tiny", "--layers", "1", "--output", path, "--device", "cpu"]) == 0
    argv = ["run", "-m", path, "--device", "cpu", "--prompt-ids", ",".join(str(i) for i in range(5, 45)),
            "--max-tokens", "3", "--temperature", "0", "--prompt-cache", pc]
    assert main(argv) == 0
    st = load_session(pc)
    assert st["tokens"].tolist() == list(range(5, 45))
    with caplog.at_level(logging.INFO, logger="barq"):
        assert main(argv) == 0
    assert any("40 tokens reusable" in r.getMessage() for r in caplog.records)
