"""Mixture-of-experts FFN block (Mixtral, Qwen-MoE, DeepSeek-V2 routed + shared experts).

Parity: ``MoELayer`` / ``FusedMoE`` (``models/src/moe_fused.rs:95-308``: gate softmax, top-k, SER
drop of experts whose gate weight is below a threshold, per-expert SwiGLU FFN, weighted sum) and
the DeepSeek routing in ``models/src/deepseek.rs:140-163``.  The reference runs experts token by
token on the CPU; here the whole layer stays on the device:

    router logits (small matmul) -> moe_route (gate, group-limited top-k, renorm, SER, counts,
    offsets, dispatch of token rows into expert-major order) -> grouped tcgen05 GEMM over the
    stacked gate|up experts with the SwiGLU epilogue -> grouped GEMM over the stacked down experts
    whose epilogue stores gate_weight * y per sorted row -> moe_combine, which adds each token's
    rows into the residual stream in slot order (deterministic: no floating-point atomics).

No step depends on host-side expert counts, so MoE decode steps are CUDA-graph capturable.
``fused=False`` (the CLI's ``--fmoe off``) runs the experts one by one instead, as the baseline.
"""
from __future__ import annotations

import torch

from .. import ops
from ..ops import EPI_ADD_F32, EPI_MOE_COMBINE, EPI_SWIGLU_Q8, QWeight
from .config import ModelConfig
from .weights import PackedTensor


def _dense(pt: PackedTensor, device) -> torch.Tensor:
    from .reference import dequant_tensor

    return dequant_tensor(pt).reshape(pt.shape).to(device, torch.float32).contiguous()


def _qw(pt: PackedTensor, device) -> QWeight:
    return QWeight.from_packed(pt.data, pt.ggml_type, pt.rows, pt.cols, device)


class MoEBlock:
    def __init__(self, cfg: ModelConfig, tensors: dict[str, PackedTensor], prefix: str, device, expert0: int = 0):
        self.cfg = cfg
        self.device = device
        self.E, self.k = cfg.n_experts, cfg.n_experts_used
        # expert parallel: this block holds experts [expert0, expert0 + E_local) of the E routed ones
        self.e0 = expert0
        self.E_local = tensors[prefix + "ffn_gate_exps.weight"].shape[0]
        self.F = cfg.expert_ffn
        self.router = _dense(tensors[prefix + "ffn_gate_inp.weight"], device)  # [E, H]
        g = _qw(tensors[prefix + "ffn_gate_exps.weight"], device)  # E*F rows
        u = _qw(tensors[prefix + "ffn_up_exps.weight"], device)
        self.down = _qw(tensors[prefix + "ffn_down_exps.weight"], device)  # E*H rows, K = F
        if g.wtype == ops.W_BF16 or self.F % 64:
            raise ValueError("MoE experts need a quantized type and an expert width that is a multiple of 64")
        self.gate_up = ops.interleave_gate_up(g, u).finalize()  # per expert: 2F contiguous rows
        self.down.finalize()
        self.shared = None
        if cfg.n_shared_experts:
            sg = _qw(tensors[prefix + "ffn_gate_shexp.weight"], device)
            su = _qw(tensors[prefix + "ffn_up_shexp.weight"], device)
            sd = _qw(tensors[prefix + "ffn_down_shexp.weight"], device)
            self.shared = (ops.interleave_gate_up(sg, su).finalize(), sd.finalize())
        self.sigmoid = cfg.expert_gating == "sigmoid"
        self.renorm = cfg.arch != "deepseek2" or cfg.expert_weights_norm
        # tensor parallel with replicated shared experts: only one rank adds their output to the
        # partial sums the all-reduce completes
        self.shared_here = True
        self.stats = {"tokens": 0, "dispatched": 0}
        self.load = None  # models.moe_stats.ExpertLoad when expert-load counting is on
        self.layer_index = 0

    # ------------------------------------------------------------------ forward
    def forward(self, runner, hq, hb: torch.Tensor, T: int, x: torch.Tensor) -> None:
        """Adds the MoE FFN output of the normalized activations ``hb`` [T, H] into ``x`` (f32)."""
        ser = getattr(runner, "ser_threshold", 0.0)
        logits = ops.router_logits(hb, self.router)  # [T, E] f32
        if getattr(runner, "fused_moe", True):
            self._fused(logits, hb, T, x, ser)
        else:
            self._unfused(logits, hb, T, x, ser)
        if self.shared is not None and self.shared_here:
            gu, down = self.shared
            if T <= 8 and hq is not None:
                h2 = ops.gemv(gu, hq, T, EPI_SWIGLU_Q8, x2=runner.x2)
                ops.gemv(down, h2, T, EPI_ADD_F32, out=x, x2=runner.x2)
            else:
                h = ops.gemm(gu, hb, EPI_SWIGLU_Q8)
                ops.gemm(down, h, EPI_ADD_F32, out=x)

    def _route_args(self, ser: float) -> dict:
        cfg = self.cfg
        return dict(sigmoid=self.sigmoid, renorm=self.renorm, n_group=max(1, cfg.n_expert_groups),
                    topk_group=max(1, cfg.n_group_used),
                    ser_threshold=ser, scale=cfg.expert_weights_scale)

    def _fused(self, logits, hb, T, x, ser):
        r = ops.MoeRouting(T, self.E, self.k, hb.shape[1], hb.dtype, self.device)
        ops.moe_route(logits, hb, self.k, r, **self._route_args(ser))
        # rows are sorted by expert: the local experts' rows are the window off[e0 .. e0 + E_local]
        off = r.off[self.e0:self.e0 + self.E_local + 1]
        if self.load is not None:  # rows routed to each of the E experts (sorted-row offsets)
            self.load.add(self.layer_index, r.off[1:self.E + 1] - r.off[:self.E])
        h = ops.gemm_grouped(self.gate_up, r.xs, off, self.E_local, EPI_SWIGLU_Q8)  # [T*k, F]
        ys = ops.gemm_grouped(self.down, h, off, self.E_local, EPI_MOE_COMBINE, row_tok=r.row_tok, row_w=r.row_w)
        ops.moe_combine(ys, r, T, off[0:1], off[self.E_local:self.E_local + 1], x)

    def _unfused(self, logits, hb, T, x, ser):
        """Baseline: route on the device, then one expert at a time (host-side token lists)."""
        r = ops.MoeRouting(T, self.E, self.k, hb.shape[1], hb.dtype, self.device)
        ops.moe_route(logits, hb, self.k, r, **self._route_args(ser))
        ids, wts = r.ids[:T].cpu(), r.weights[:T].cpu()
        for e in range(self.E_local):
            sel = (ids == self.e0 + e) & (wts > 0)
            if not bool(sel.any()):
                continue
            tok = sel.nonzero()[:, 0]
            wt = wts[sel].to(self.device)
            tok_d = tok.to(self.device)
            ge = self.gate_up.row_slice(e * 2 * self.F, 2 * self.F)
            de = self.down.row_slice(e * x.shape[1], x.shape[1])
            h = ops.gemm(ge, hb.index_select(0, tok_d).contiguous(), EPI_SWIGLU_Q8)
            y = ops.gemm(de, h, ops.EPI_STORE_F32)
            x.index_add_(0, tok_d, y * wt[:, None])
