"""Basic usage: greedy and sampled generation, streaming, chat, batch.

    python examples/basic_inference.py [model.gguf]
"""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from barq_inference_b200.client import Client, GenerationConfig  # noqa: E402
from simple_inference import demo_model  # noqa: E402

if __name__ == "__main__":
    client = Client.from_gguf(sys.argv[1] if len(sys.argv) > 1 else demo_model())

    print("1. greedy:", client.generate("Once upon a time", GenerationConfig(max_tokens=16, temperature=0)).text)

    cfg = GenerationConfig(max_tokens=16, temperature=0.8, top_k=40, top_p=0.95, seed=7)
    print("2. sampled:", client.generate("Once upon a time", cfg).text)

    print("3. streaming: ", end="")
    for piece in client.stream("The model is fast", GenerationConfig(max_tokens=16, temperature=0)):
        print(piece, end="", flush=True)
    print()

    r = client.chat([{"role": "system", "content": "You are terse."},
                     {"role": "user", "content": "Say hello."}], GenerationConfig(max_tokens=16, temperature=0))
    print("4. chat:", r.text)

    for i, r in enumerate(client.generate_batch(["the", "and the", "hello world"], GenerationConfig(max_tokens=8))):
        print(f"5. batch[{i}]:", r.text)
