"""Advanced usage: JSON mode, JSON schema, a custom GBNF grammar, stop strings, penalties.

    python examples/advanced_inference.py [model.gguf]
"""
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from barq_inference_b200.client import Client, GenerationConfig  # noqa: E402
from simple_inference import demo_model  # noqa: E402

if __name__ == "__main__":
    client = Client.from_gguf(sys.argv[1] if len(sys.argv) > 1 else demo_model())

    schema = {"type": "object", "properties": {"name": {"type": "string"}, "age": {"type": "integer"}},
              "required": ["name", "age"]}
    r = client.generate("Generate a user profile in JSON:", GenerationConfig(max_tokens=48, json_schema=schema, seed=1))
    print("1. JSON schema:", r.text, f"(finish: {r.finish_reason})")
    if r.finish_reason == "stop":
        print("   parsed:", json.loads(r.text))

    r = client.generate("Any JSON:", GenerationConfig(max_tokens=32, json_mode=True, seed=2))
    print("2. JSON mode:", r.text)

    yes_no = 'root ::= ("yes" | "no") "."\n'
    print("3. grammar:", client.generate("Is it fast?", GenerationConfig(max_tokens=8, grammar=yes_no)).text)

    cfg = GenerationConfig(max_tokens=32, temperature=0.7, repetition_penalty=1.2, presence_penalty=0.5, stop=["."])
    print("4. stop + penalties:", client.generate("List things:", cfg).text)
