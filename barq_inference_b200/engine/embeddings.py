"""Sentence embeddings from a decoder: the final-norm hidden states of a prompt, mean-pooled over
its positions and L2-normalised.

Parity: ``ContextParams::embeddings`` (``models/src/context.rs:62``, "enable embeddings extraction"),
a flag the reference defines and never reads.  Here ``Engine.embed`` / ``CPUEngine.embed`` produce
the vectors and the HTTP server exposes them as ``POST /v1/embeddings``.

GPU engine: each prompt runs as prefill chunks through the model runner on pages borrowed from
the KV pool (returned afterwards); the runner copies every row's final residual stream into a
caller buffer (``StepInput.hidden_out``) before its head, and the output norm and the pooling run
here.  Single-GPU runners of the dense and MoE families (not MLA, not tensor / pipeline parallel).
"""
from __future__ import annotations

import numpy as np
import torch


def _pool(h_sum: torch.Tensor, n: int, normalize: bool) -> torch.Tensor:
    e = h_sum / max(1, n)
    if normalize:
        e = e / e.norm().clamp_min(1e-12)
    return e


def embed_cpu(engine, prompts: list[list[int]], normalize: bool = True) -> torch.Tensor:
    out = []
    with torch.no_grad():
        for p in prompts:
            if not p:
                raise ValueError("empty input")
            h = engine.model.forward(list(p), {}, hidden=True)  # [T, hidden], final norm applied
            out.append(_pool(h.sum(0), len(p), normalize))
    return torch.stack(out)


def embed_gpu(engine, prompts: list[list[int]], normalize: bool = True) -> torch.Tensor:
    from ..models.runner import LlamaRunner, StepInput

    runner, ec, cfg = engine.runner, engine.ecfg, engine.cfg
    if not isinstance(runner, LlamaRunner) or runner.pp is not None or (runner.comm is not None and runner.comm.world > 1):
        raise NotImplementedError("embeddings: single-GPU dense / MoE runners only")
    bs = engine.blocks.block_size
    dev = engine.device
    out = []
    with torch.no_grad():
        for p in prompts:
            n = len(p)
            if n == 0:
                raise ValueError("empty input")
            if n >= ec.max_model_len:
                raise ValueError(f"input of {n} tokens exceeds max_model_len {ec.max_model_len}")
            nb = engine.blocks.blocks_for(n)
            if not engine.blocks.can_allocate(nb) and engine.prefix_cache is not None:
                engine.prefix_cache.evict(nb - engine.blocks.n_free)
            blocks = engine.blocks.allocate(nb)
            try:
                tbl = np.asarray(blocks, np.int64)
                acc = torch.zeros(cfg.hidden, dtype=torch.float32, device=dev)
                step = max(1, ec.max_num_batched_tokens)
                for c0 in range(0, n, step):
                    c1 = min(n, c0 + step)
                    T = c1 - c0
                    pos = np.arange(c0, c1, dtype=np.int64)
                    slots = tbl[pos // bs] * bs + pos % bs
                    hid = torch.empty(T, cfg.hidden, dtype=torch.float32, device=dev)
                    d = lambda a, dt: torch.as_tensor(a, dtype=dt).to(dev)  # noqa: E731
                    inp = StepInput(d(np.asarray(p[c0:c1]), torch.int32), d(pos, torch.int32), d(slots, torch.int64),
                                    d(tbl[None, :], torch.int32), d([c1], torch.int32), d([T - 1], torch.int64),
                                    False, q_start=d([0, T], torch.int32), max_q=T, hidden_out=hid)
                    runner.forward(inp)
                    h = hid * torch.rsqrt(hid.pow(2).mean(-1, keepdim=True) + cfg.rms_eps) * runner.out_norm
                    acc += h.sum(0)
                out.append(_pool(acc, n, normalize).cpu())
            finally:
                engine.blocks.release(blocks)
    return torch.stack(out)
