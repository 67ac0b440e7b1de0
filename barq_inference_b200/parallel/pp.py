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
    """This rank's pipeline stage.  With tensor parallelism inside each stage (``tp`` > 1) the
    global rank of (stage s, tensor rank t) is ``s * tp + t``: hidden states go to the rank with the
    same tensor rank in the next stage, and the last stage's rank broadcasts the (already gathered)
    logits over ``group``, the ranks sharing this tensor rank."""
    stage: int
    world: int
    l0: int
    l1: int
    tp: int = 1
    tp_rank: int = 0
    group: object = None

    @property
    def is_last(self) -> bool:
        return self.stage == self.world - 1

    def global_rank(self, stage: int) -> int:
        return stage * self.tp + self.tp_rank

    def send(self, x: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.send(x.contiguous(), self.global_rank(self.stage + 1))

    def recv(self, x: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.recv(x, self.global_rank(self.stage - 1))

    def broadcast_logits(self, logits: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.broadcast(logits, self.global_rank(self.world - 1), group=self.group)


def grid_groups(tp: int, pp: int):
    """Process groups of a tp x pp grid (global rank = stage * tp + tensor rank): returns
    (stage, tensor rank, this rank's tensor-parallel group, this rank's pipeline group).  Every
    rank creates every group, in the same order, as ``new_group`` requires."""
    import torch.distributed as dist

    rank, world = dist.get_rank(), dist.get_world_size()
    if world != tp * pp:
        raise ValueError(f"tp={tp} x pp={pp} needs {tp * pp} ranks, the process group has {world}")
    stage, t = divmod(rank, tp)
    tp_group = pp_group = None
    for s in range(pp):
        g = dist.new_group([s * tp + i for i in range(tp)])
        if s == stage:
            tp_group = g
    for i in range(tp):
        g = dist.new_group([s * tp + i for s in range(pp)])
        if i == t:
            pp_group = g
    return stage, t, tp_group, pp_group
