"""Smallest program: load a GGUF model and complete a prompt.

    python examples/simple_inference.py model.gguf "The capital of France is"

Without arguments it writes a small random-init model first (no download needed), so the output
is gibberish but every step runs.
"""
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from barq_inference_b200.client import Client, GenerationConfig  # noqa: E402


def demo_model() -> str:
    from barq_inference_b200.cli import main

    path = os.path.join(tempfile.gettempdir(), "barq-demo-tiny.gguf")
    if not os.path.exists(path):
        main(["make-random-gguf", "--arch", "tiny", "--layers", "2", "--output", path, "--device", "cpu"])
    return path


if __name__ == "__main__":
    model = sys.argv[1] if len(sys.argv) > 1 else demo_model()
    prompt = sys.argv[2] if len(sys.argv) > 2 else "Hello, my name is"
    client = Client.from_gguf(model)
    r = client.generate(prompt, GenerationConfig(max_tokens=24, temperature=0.0))
    print(prompt + r.text)
    print(f"[{len(r.tokens)} tokens, {r.tokens_per_second:.1f} tok/s, finish: {r.finish_reason}]")
