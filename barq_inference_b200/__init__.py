"""barq_inference_b200: a Blackwell (sm_100a) native GGUF LLM inference engine."""
__version__ = "0.1.0"
