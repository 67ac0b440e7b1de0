"""The reference's end-to-end CLI fixture, rebuilt as a GGUF file: a 0-layer LLaMA with hidden 4 and
a 128-token vocabulary where token_embd[2] = e0 and output[3] = 10 * e0, so the prompt "hello"
(token 2; given as ids: the fixture vocabulary has no intermediate SentencePiece pieces to merge
characters into "▁hello") is continued by token 3 ("world") (``cli/tests/integration/fixtures.rs:13-66``,
``end_to_end.rs:25-38``).  Run through this package's CLI on the CPU engine."""
import os
import subprocess
import sys

import numpy as np

from barq_inference_b200.gguf import GGMLType, GGUFWriter

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _fixture(path):
    V, H = 128, 4
    toks = ["<unk>", "<s>", "▁hello", "▁world"] + [f"<t{i}>" for i in range(4, V)]
    emb = np.zeros((V, H), np.float32)
    emb[2, 0] = 1.0
    out = np.zeros((V, H), np.float32)
    out[3, 0] = 10.0
    w = GGUFWriter(path, arch="llama")
    for k, v in {"llama.block_count": 0, "llama.embedding_length": H, "llama.attention.head_count": 1,
                 "llama.attention.head_count_kv": 1, "llama.feed_forward_length": 8, "llama.context_length": 64,
                 "llama.attention.layer_norm_rms_epsilon": 1e-5, "tokenizer.ggml.model": "llama",
                 "tokenizer.ggml.tokens": toks, "tokenizer.ggml.scores": [0.0] * V,
                 "tokenizer.ggml.token_type": [2, 3] + [1] * (V - 2), "tokenizer.ggml.bos_token_id": 1,
                 "tokenizer.ggml.eos_token_id": 0, "tokenizer.ggml.add_bos_token": False}.items():
        w.add(k, v)
    w.add_tensor("token_embd.weight", emb, GGMLType.F32, (V, H))
    w.add_tensor("output.weight", out, GGMLType.F32, (V, H))
    w.add_tensor("output_norm.weight", np.ones(H, np.float32), GGMLType.F32, (H,))
    w.write()


def test_hello_world_fixture(tmp_path):
    path = str(tmp_path / "fixture.gguf")
    _fixture(path)
    r = subprocess.run([sys.executable, "-m", "barq_inference_b200.cli", "run", "-m", path, "--device", "cpu",
                        "--prompt-ids", "2", "--max-tokens", "1", "--temperature", "0"], cwd=ROOT, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().endswith("world"), r.stdout
