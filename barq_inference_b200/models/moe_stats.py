"""Expert-load statistics of MoE routing: per-layer token counts per expert and balance measures.

Parity: ``MoERouter::compute_aux_loss`` (``advanced/src/moe.rs:73-82``: ``coef * variance(counts)``
over experts) — there computed from counts the caller supplies; here the counts come from the
routing the model actually ran.  Counting is off unless enabled (``BARQ_MOE_STATS=1`` or
``enable(model)``) so the default decode graph gains no launches: when on, the device MoE block
adds the per-expert row counts of each routing (the difference of the routing kernel's expert
offsets, one small device op) into a device counter; the fp32 reference forward counts on the CPU.
"""
from __future__ import annotations

import os

import torch


class ExpertLoad:
    def __init__(self, n_layers: int, n_experts: int, device="cpu"):
        self.counts = torch.zeros(n_layers, n_experts, dtype=torch.int64, device=device)

    def add(self, layer: int, per_expert: torch.Tensor) -> None:
        self.counts[layer] += per_expert.to(self.counts.device, torch.int64)

    def reset(self) -> None:
        self.counts.zero_()

    def summary(self, aux_loss_coef: float = 0.01) -> dict:
        """Totals and balance measures over the routed layers: ``aux_loss`` is the reference's
        ``coef * mean((c - mean(c))^2)`` per layer, averaged; ``max_over_mean`` the hottest expert's
        load relative to a perfectly even split; ``cv`` the coefficient of variation."""
        c = self.counts.double().cpu()
        used = c.sum(1) > 0
        if not bool(used.any()):
            return {"tokens_routed": 0, "aux_loss": 0.0, "max_over_mean": 0.0, "cv": 0.0, "per_layer": []}
        c = c[used]
        mean = c.mean(1, keepdim=True)
        var = ((c - mean) ** 2).mean(1)
        return {
            "tokens_routed": int(c.sum()),
            "aux_loss": float((aux_loss_coef * var).mean()),
            "max_over_mean": float((c.max(1).values / mean[:, 0]).mean()),
            "cv": float((var.sqrt() / mean[:, 0]).mean()),
            "per_layer": c.long().tolist(),
        }


def enabled_by_env() -> bool:
    return os.environ.get("BARQ_MOE_STATS", "0") not in ("0", "", "false")


def enable(model, device=None) -> ExpertLoad:
    """Attach an ``ExpertLoad`` to a runner (its MoE blocks) or a ``ReferenceModel``."""
    cfg = model.cfg
    load = ExpertLoad(cfg.n_layers, max(1, cfg.n_experts), device or getattr(model, "device", "cpu"))
    model.expert_load = load
    for i, L in enumerate(getattr(model, "layers", []) or []):
        moe = getattr(L, "moe", None)
        if moe is not None:
            moe.load, moe.layer_index = load, i
    return load
