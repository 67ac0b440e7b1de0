"""Pipeline parallelism: contiguous layer stages, one process per GPU.

Parity: ``PipelineParallel::{forward_pipeline,schedule_microbatches}``
(``backend/src/cuda_multi_gpu.rs:332-398``: a layer range per stage, activations passed from stage
to stage; Unsupported in the reference).  Here stage s runs layers [l0, l1) of the model; stage 0
also embeds, the last stage also holds the output norm and head.  Per forward, the hidden states
[T, H] (f32) go from stage to stage with NCCL send/recv, and the last stage broadcasts the logits so
that every rank's (replicated) scheduler and sampler stay in step.  Only the tensors of a rank's
own layers are uploaded to its GPU.  On one NVSwitch node tensor parallelism is the faster way to
use several GPUs; pipeline stages are for models whose weights do not fit one GPU with TP alone.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.weights import PackedTensor


def stage_layers(n_layers: int, world: int) -> list[tuple[int, int]]:
    """Contiguous layer ranges, sizes differing by at most one (earlier stages take the extra)."""
    if world > n_layers:
        raise ValueError(f"pipeline: {world} stages for {n_layers} layers")
    base, extra = divmod(n_layers, world)
    out, l0 = [], 0
    for s in range(world):
        n = base + (1 if s < extra else 0)
        out.append((l0, l0 + n))
        l0 += n
    return out


def shard_pp(tensors: dict[str, PackedTensor], n_layers: int, stage: int, world: int) -> dict[str, PackedTensor]:
    """The tensors stage ``stage`` needs: its layers, embeddings on stage 0, norm + head on the last."""
    l0, l1 = stage_layers(n_layers, world)[stage]
    last = stage == world - 1
    out = {}
    for name, pt in tensors.items():
        if name.startswith("blk."):
            i = int(name.split(".")[1])
            if l0 <= i < l1:
                out[name] = pt
        elif name == "token_embd.weight":
            if stage == 0 or (last and "output.weight" not in tensors):  # tied head
                out[name] = pt
        elif name in ("output.weight", "output_norm.weight"):
            if last:
                out[name] = pt
        else:
            out[name] = pt
    return out


@dataclass
class PPInfo:
    stage: int
    world: int
    l0: int
    l1: int

    @property
    def is_last(self) -> bool:
        return self.stage == self.world - 1

    def send(self, x: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.send(x.contiguous(), self.stage + 1)

    def recv(self, x: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.recv(x, self.stage - 1)

    def broadcast_logits(self, logits: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.broadcast(logits, self.world - 1)
