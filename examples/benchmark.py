"""Throughput of a batch of prompts through the client API (end to end, host included).

    python examples/benchmark.py [model.gguf] [batch] [max_tokens]

For the device-timed headline benchmark use ``bench.py`` / ``barq benchmark``.
"""
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from barq_inference_b200.client import Client, GenerationConfig  # noqa: E402
from simple_inference import demo_model  # noqa: E402

if __name__ == "__main__":
    client = Client.from_gguf(sys.argv[1] if len(sys.argv) > 1 else demo_model())
    batch = int(sys.argv[2]) if len(sys.argv) > 2 else 4
    n = int(sys.argv[3]) if len(sys.argv) > 3 else 16
    cfg = GenerationConfig(max_tokens=n, temperature=0.0)
    client.generate("warm up", GenerationConfig(max_tokens=2))
    t0 = time.perf_counter()
    res = client.generate_batch([f"prompt number {i}:" for i in range(batch)], cfg)
    dt = time.perf_counter() - t0
    toks = sum(len(r.tokens) for r in res)
    print(f"{batch} prompts, {toks} tokens in {dt:.2f} s: {toks / dt:.1f} tok/s aggregate")
