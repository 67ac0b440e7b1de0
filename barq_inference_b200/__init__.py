"""barq_inference_b200: a Blackwell (sm_100a) native GGUF LLM inference engine.

Top-level names load on first use: ``Client``, ``GenerationConfig`` (text API), ``RemoteClient``
(the same API against a running HTTP server), ``Engine``,
``EngineConfig``, ``SamplingParams``, ``ModelContext`` (token API), ``read_gguf``.
"""
__version__ = "0.1.0"

_LAZY = {
    "Client": ("client", "Client"),
    "GenerationConfig": ("client", "GenerationConfig"),
    "RemoteClient": ("remote", "RemoteClient"),
    "Engine": ("engine.engine", "Engine"),
    "EngineConfig": ("engine.engine", "EngineConfig"),
    "SamplingParams": ("engine.sampling_params", "SamplingParams"),
    "ModelContext": ("engine.context", "ModelContext"),
    "read_gguf": ("gguf", "read_gguf_split"),
}


def __getattr__(name):
    if name in _LAZY:
        import importlib

        mod, attr = _LAZY[name]
        return getattr(importlib.import_module(f".{mod}", __name__), attr)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
