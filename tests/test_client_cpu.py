"""The high-level client API and the shipped examples, on the CPU engine with a random-init model."""
import json
import os
import subprocess
import sys

import pytest

from barq_inference_b200.client import Client, GenerationConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    from barq_inference_b200.cli import main

    path = str(tmp_path_factory.mktemp("m") / "tiny.gguf")
    assert main(["make-random-gguf", "--arch", "tiny", "--layers", "1", "--output", path, "--device", "cpu"]) == 0
    return path


def test_generate_stream_batch_agree(model):
    c = Client.from_gguf(model, device="cpu")
    cfg = GenerationConfig(max_tokens=8, temperature=0.0)
    r = c.generate("hello world", cfg)
    assert r.prompt_tokens > 0 and 0 < len(r.tokens) <= 8 and r.latency_s > 0
    assert "".join(c.stream("hello world", cfg)) == r.text
    b = c.generate_batch(["hello world", "the model"], cfg)
    assert b[0].text == r.text and b[0].tokens == r.tokens


def test_stop_strings_and_json(model):
    c = Client.from_gguf(model, device="cpu")
    r = c.generate("hello", GenerationConfig(max_tokens=24, temperature=0.0))
    if len(r.text) > 2:
        stop = r.text[1:3]
        r2 = c.generate("hello", GenerationConfig(max_tokens=24, temperature=0.0, stop=[stop]))
        assert stop not in r2.text and r.text.startswith(r2.text) and r2.finish_reason == "stop"
    j = c.generate("json:", GenerationConfig(max_tokens=64, json_mode=True, seed=3))
    if j.finish_reason == "stop":
        json.loads(j.text)
    r3 = c.chat([{"role": "user", "content": "hi"}], GenerationConfig(max_tokens=4, temperature=0.0))
    assert len(r3.tokens) <= 4


@pytest.mark.parametrize("script", ["simple_inference.py", "basic_inference.py", "advanced_inference.py",
                                    "benchmark.py"])
def test_examples_run(model, script):
    r = subprocess.run([sys.executable, os.path.join(ROOT, "examples", script), model], cwd=ROOT,
                       capture_output=True, text=True, timeout=300, env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert r.returncode == 0, r.stderr[-2000:]
