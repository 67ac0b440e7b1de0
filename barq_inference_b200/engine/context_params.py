"""``ContextParams``: the llama.cpp-style context knobs, mapped onto this engine's configuration.

Parity: ``ContextParams`` and its presets ``gpu_optimized`` / ``cpu_optimized`` / ``quality`` /
``speed`` (``models/src/context.rs:47-162``).  The reference defines these fields but most of them
steer nothing (``type_k``/``type_v`` are never read by its KV cache, ``flash_attn`` and the thread
counts only annotate).  Here every field either sets an engine switch or is documented as having
no effect on this design:

* ``n_ctx`` -> ``EngineConfig.max_model_len`` (0 = the model's trained context)
* ``n_batch`` -> ``max_num_batched_tokens`` (token budget of one engine step)
* ``n_ubatch`` -> the prefill chunk: the scheduler's step budget is ``min(n_batch, n_ubatch)``
* ``n_seq_max`` -> ``max_num_seqs`` (continuous-batching width)
* ``type_k`` / ``type_v`` (ggml type ids) -> ``kv_dtype``: F16 -> fp16, BF16 -> bf16, any 8-bit or
  smaller type (Q8_0, Q4_0, ...) -> fp8 e4m3 (the narrowest KV format the attention kernels
  read); K and V share one dtype, the narrower of the two wins
* ``n_gpu_layers`` -> 0 selects the CPU engine; any other value offloads every layer (partial
  offload is not a mode of this engine: the GPU path holds the whole model)
* ``rope_freq_base`` / ``rope_freq_scale`` -> model overrides (``rope_theta``; a scale below 1
  is linear position interpolation, factor ``1/scale``); 0 keeps the GGUF value
* ``flash_attn`` -> always on (the paged attention kernels are flash-style); recorded only
* ``defrag_thold`` -> no effect: the paged KV pool has no fragmentation to compact (sequences
  own whole 16-token pages through block tables)
* ``n_threads`` / ``n_threads_batch`` -> torch CPU threads of the CPU engine
* ``embeddings`` -> recorded (hidden-state extraction is not an engine output)
"""
from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass

# ggml type ids (public GGUF spec) that name K/V cache formats
_F32, _F16, _Q4_0, _Q8_0, _BF16 = 0, 1, 2, 8, 30


@dataclass
class ContextParams:
    n_ctx: int = 8192
    n_batch: int = 512
    n_threads: int = 4
    n_threads_batch: int = 4
    rope_scaling_type: int = 0
    rope_freq_base: float = 0.0
    rope_freq_scale: float = 0.0
    embeddings: bool = False
    flash_attn: bool = True
    n_gpu_layers: int = 9999
    type_k: int = _F16
    type_v: int = _F16
    defrag_thold: float = 0.1
    n_ubatch: int = 512
    n_seq_max: int = 32

    # ------------------------------------------------------------------ presets
    @staticmethod
    def gpu_optimized() -> "ContextParams":
        return ContextParams(n_ctx=8192, n_gpu_layers=9999, flash_attn=True, n_seq_max=64, n_batch=8192,
                             n_ubatch=8192)

    @staticmethod
    def cpu_optimized() -> "ContextParams":
        n = max(1, (os.cpu_count() or 2) // 2)
        return ContextParams(n_threads=n, n_threads_batch=n, flash_attn=False, n_gpu_layers=0)

    @staticmethod
    def quality() -> "ContextParams":
        """Widest KV format: bf16 keys and values."""
        return ContextParams(type_k=_BF16, type_v=_BF16)

    @staticmethod
    def speed() -> "ContextParams":
        """8-bit (fp8) KV and a 4096-token context."""
        return ContextParams(type_k=_Q8_0, type_v=_Q8_0, n_ctx=4096)

    # ------------------------------------------------------------------ mapping
    def kv_dtype(self) -> str:
        def one(t: int) -> tuple[int, str]:
            if t in (_F32, _F16):
                return 16, "fp16"
            if t == _BF16:
                return 16, "bf16"
            return 8, "fp8"

        (bk, k), (bv, v) = one(self.type_k), one(self.type_v)
        return "fp8" if min(bk, bv) == 8 else k  # fp16 vs bf16 for K and V: K's choice

    @property
    def use_gpu(self) -> bool:
        return self.n_gpu_layers != 0

    def model_overrides(self) -> dict:
        ov: dict = {}
        if self.rope_freq_base > 0:
            ov["rope_theta"] = float(self.rope_freq_base)
        if 0 < self.rope_freq_scale < 1:
            ov["rope_scaling"] = "linear"
            ov["rope_factor"] = 1.0 / float(self.rope_freq_scale)
        return ov

    def apply_to_model(self, cfg):
        """A copy of ``cfg`` with the context's RoPE overrides and context length applied."""
        ov = self.model_overrides()
        if self.n_ctx > 0:
            ov["max_ctx"] = min(cfg.max_ctx, self.n_ctx) if cfg.max_ctx else self.n_ctx
        return dataclasses.replace(cfg, **ov)

    def engine_config(self, model_max_ctx: int = 0, **kw):
        """The ``EngineConfig`` these parameters select (GPU engine)."""
        from .engine import EngineConfig

        n_ctx = self.n_ctx or model_max_ctx or 4096
        if model_max_ctx:
            n_ctx = min(n_ctx, model_max_ctx)
        step = max(1, min(self.n_batch, self.n_ubatch))
        base = dict(max_model_len=n_ctx, max_num_batched_tokens=step, max_num_seqs=max(1, self.n_seq_max),
                    kv_dtype=self.kv_dtype(), chunked_prefill=True)
        base.update(kw)
        return EngineConfig(**base)

    def make_engine(self, cfg, tensors, device: str | None = None, **kw):
        """Builds the engine these parameters select: the CPU engine for ``n_gpu_layers == 0``,
        else the CUDA engine on ``device`` (default ``cuda``)."""
        cfg = self.apply_to_model(cfg)
        if not self.use_gpu:
            import torch

            from .cpu_engine import CPUEngine

            torch.set_num_threads(max(1, self.n_threads))
            return CPUEngine(cfg, tensors, max_model_len=cfg.max_ctx)
        from .engine import Engine

        return Engine(cfg, tensors, self.engine_config(cfg.max_ctx, device=device or "cuda", **kw))
