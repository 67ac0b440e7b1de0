"""DeepSeek-V2 (Lite) runner: multi-head latent attention over a paged latent cache + MoE FFNs.

Parity: ``DeepSeekModel`` (``models/src/deepseek.rs:55-163``: MLA projections with ``kv_lora_rank``,
rope/nope split, shared + routed experts, first ``n_dense_layers`` dense) and the ``--mla`` flag
(``cli/src/main.rs:507-525``).  The reference computes none of the MLA attention; here:

* the KV cache holds one 576-wide row per token and layer: the RMS-normalized latent ``c`` (512)
  and the shared rotary key ``k_pe`` (64) -- 8x less cache than materialized per-head K/V;
* queries are absorbed: ``q_lat = q_nope . W_UK`` (per-head 128x512 blocks of ``attn_kv_b``), so the
  attention kernel (K10, ``csrc/kernels/mla.cu``) scores ``q_lat . c + q_pe . k_pe`` directly on the
  cached latents and returns ``o_lat = softmax . c``; ``o_lat . W_UV^T`` gives the head outputs.
  Both absorptions run as grouped tcgen05 GEMMs (one group per head, Q8_0 weights, bf16
  activations) -- no cuBLAS on the attention path;
* expert FFNs are :class:`MoEBlock` (group-limited top-k, shared experts), the first layer is dense;
* tensor parallel (``tp`` / ``comm``): each rank holds the query projection, W_UK / W_UV and the
  output-projection columns of H / tp heads, the latent path (q_a, kv_a, cache) replicated; the
  attention kernel runs the 16-head layout with this rank's heads in place (the others' queries
  zero, their outputs unused), and the output projection's partial sums are all-reduced like the
  dense models' row-parallel layers.  Experts are split by expert.

Activations in the tensor-core GEMMs are bf16 (DeepSeek overflows fp16).
"""
from __future__ import annotations

import math

import torch

from .. import ops
from ..ops import EPI_ADD_F32, EPI_STORE_F32, EPI_SWIGLU_Q8
from .config import ModelConfig
from .moe import MoEBlock
from .rope import attn_scale, rope_cos_sin
from .runner import GEMV_MAX_T, Layer, LlamaRunner, StepInput, _f32, _qw, apply_embed_overrides
from .weights import PackedTensor

LAT, ROPE = 512, 64


def _q8_grouped(w: torch.Tensor, dev) -> ops.QWeight:
    """f32 [rows, K] -> Q8_0 QWeight on ``dev`` (rows are whole 128-row groups of a grouped GEMM)."""
    from ..gguf import GGMLType, quantize

    w = w.to(dev).contiguous()
    return ops.QWeight.from_packed(quantize(w, GGMLType.Q8_0), GGMLType.Q8_0, w.shape[0], w.shape[1], dev).finalize()


class DeepseekV2Runner(LlamaRunner):
    def __init__(self, cfg: ModelConfig, tensors: dict[str, PackedTensor], device="cuda",
                 kv_dtype: torch.dtype = torch.bfloat16, ser_threshold: float = 0.0, act_x2: bool = True,
                 tp=None, comm=None):
        if cfg.kv_lora_rank != LAT or cfg.qk_rope_dim != ROPE or cfg.n_heads != 16:
            raise ValueError("DeepseekV2Runner: the MLA kernel is built for 16 heads, latent 512, rope 64")
        if kv_dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("DeepseekV2Runner: the latent KV cache is float16 or bfloat16 (no fp8 MLA kernel)")
        from .reference import dequant_tensor

        self.cfg = cfg
        self.tp, self.comm, self.pp = tp, comm, None
        self.h0 = tp.head0 if tp is not None else 0
        self.Hl = tp.n_heads_local if tp is not None else cfg.n_heads  # heads held by this rank
        self.device = torch.device(device)
        self.kv_dtype = kv_dtype
        self.scale = attn_scale(cfg)
        self.use_gemm = None
        self.x2 = act_x2
        self.act_dtype = torch.bfloat16
        self.ser_threshold = ser_threshold
        self.fused_moe = True
        dev = self.device
        H, dn, dv = cfg.n_heads, cfg.qk_nope_dim, cfg.v_head_dim
        self.qdim = dn + ROPE
        self.embed_w = _qw(tensors["token_embd.weight"], dev)
        self.out_norm = _f32(tensors["output_norm.weight"], dev)
        self.out_w = _qw(tensors["output.weight"], dev) if "output.weight" in tensors else self.embed_w
        self.layers = []
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            L = Layer()
            L.attn_norm = _f32(tensors[p + "attn_norm.weight"], dev)
            L.ffn_norm = _f32(tensors[p + "ffn_norm.weight"], dev)
            if cfg.q_lora_rank:
                L.q_a = _qw(tensors[p + "attn_q_a.weight"], dev)
                L.q_a_norm = _f32(tensors[p + "attn_q_a_norm.weight"], dev)
                L.q_b = _qw(tensors[p + "attn_q_b.weight"], dev)
                L.wq = None
            else:
                L.wq = _qw(tensors[p + "attn_q.weight"], dev)
            L.kv_a = _qw(tensors[p + "attn_kv_a_mqa.weight"], dev)
            L.kv_a_norm = _f32(tensors[p + "attn_kv_a_norm.weight"], dev)
            kvb = dequant_tensor(tensors[p + "attn_kv_b.weight"]).view(self.Hl, dn + dv, LAT).float()
            # absorption weights as grouped tcgen05 GEMM operands (one group per head, Q8_0):
            # W_UK^T [Hl * 512, dn] maps q_nope to q_lat, W_UV [Hl * dv, 512] maps o_lat to the head outputs
            L.uk = _q8_grouped(kvb[:, :dn, :].transpose(1, 2).reshape(self.Hl * LAT, dn), dev)
            L.uv = _q8_grouped(kvb[:, dn:, :].reshape(self.Hl * dv, LAT), dev)
            L.wo = _qw(tensors[p + "attn_output.weight"], dev)
            if cfg.layer_is_moe(i):
                L.moe = MoEBlock(cfg, tensors, p, dev, expert0=tp.expert0 if tp is not None else 0)
                L.moe.shared_here = tp is None or tp.rank == 0  # shared experts are replicated under TP
            else:
                L.moe = None
                g, u = _qw(tensors[p + "ffn_gate.weight"], dev), _qw(tensors[p + "ffn_up.weight"], dev)
                L.gate_up = ops.interleave_gate_up(g, u)
                L.down = _qw(tensors[p + "ffn_down.weight"], dev)
            self.layers.append(L)
        self.cos, self.sin = rope_cos_sin(cfg, cfg.max_ctx, dev)

    # ------------------------------------------------------------------ latent KV cache
    def allocate_kv(self, num_blocks: int, block_size: int = 16):
        if block_size != 16:
            raise ValueError("MLA cache pages are 16 tokens")
        self.kv_storage = torch.zeros(self.cfg.n_layers, num_blocks, block_size, LAT + ROPE, dtype=self.kv_dtype,
                                      device=self.device)
        self.kv = [self.kv_storage[i] for i in range(self.cfg.n_layers)]
        return self.kv

    def kv_bytes_per_block(self, block_size: int = 16) -> int:
        return self.cfg.n_layers * block_size * (LAT + ROPE) * torch.finfo(self.kv_dtype).bits // 8

    # ------------------------------------------------------------------ helpers
    def _proj(self, w, hq, hb, T, mode=EPI_STORE_F32, out=None):
        if T <= GEMV_MAX_T:
            return self._lin_q8(w, hq, T, mode, out=out, xb=hb)
        return self._lin_bf16(w, hb, T, mode, out=out)

    def _norm(self, x, w, T):
        return ops.rmsnorm(x, w, self.cfg.rms_eps, want_q8=T <= GEMV_MAX_T, want_bf16=True, x2=self.x2,
                           act_dtype=self.act_dtype)

    def _per_head(self, w, x: torch.Tensor, n_out: int) -> torch.Tensor:
        """Per-head projection x [T, Hl, K] -> [T, Hl, n_out] as one grouped tcgen05 GEMM (group h =
        head h's rows of ``w``; the activations in head-major order, bf16)."""
        T, Hl, K = x.shape
        xs = x.permute(1, 0, 2).reshape(Hl * T, K).to(self.act_dtype).contiguous()
        off = torch.arange(0, (Hl + 1) * T, T, dtype=torch.int32, device=self.device)
        y = ops.gemm_grouped(w, xs, off, Hl, EPI_STORE_F32)  # [Hl * T, n_out]
        return y.view(Hl, T, n_out).permute(1, 0, 2).contiguous()

    def _dense_ffn(self, L, hq, hb, T, mode, out):
        """The leading dense FFN, replicated under tensor parallelism: rank 0 adds (or stores) it,
        the other ranks contribute zeros to the all-reduce."""
        if self.tp is not None and self.tp.rank != 0:
            if mode == EPI_STORE_F32:
                out.zero_()
            return
        if T <= GEMV_MAX_T:
            self._lin_q8(L.down, self._lin_q8(L.gate_up, hq, T, EPI_SWIGLU_Q8), T, mode, out=out)
        else:
            ops.gemm(L.down, ops.gemm(L.gate_up, hb, EPI_SWIGLU_Q8), mode, out=out)

    def _mla(self, L, li, x, inp: StepInput, T):
        cfg = self.cfg
        H = cfg.n_heads
        hb, hq = self._norm(x, L.attn_norm, T)
        if L.wq is None:
            qa = self._proj(L.q_a, hq, hb, T)
            qb, qq = ops.rmsnorm(qa, L.q_a_norm, cfg.rms_eps, want_q8=T <= GEMV_MAX_T, want_bf16=True, x2=self.x2,
                                 act_dtype=self.act_dtype)
            q = self._proj(L.q_b, qq, qb, T)
        else:
            q = self._proj(L.wq, hq, hb, T)  # f32 [T, H*qdim]
        kva = self._proj(L.kv_a, hq, hb, T)  # f32 [T, 576]
        Hl, h0 = self.Hl, self.h0
        ops.mla_kv_write(kva, L.kv_a_norm, cfg.rms_eps, self.cos, self.sin, cfg.rope_neox, inp.pos, inp.slots,
                         self.kv[li], q, Hl, self.qdim, cfg.qk_nope_dim)
        q3 = q.view(T, Hl, self.qdim)
        q_lat = self._per_head(L.uk, q3[..., :cfg.qk_nope_dim], LAT)  # [T, Hl, 512]
        if Hl != H:  # tensor parallel: this rank's heads in the kernel's 16-head layout
            ql = torch.zeros(T, H, LAT, dtype=q_lat.dtype, device=self.device)
            ql[:, h0:h0 + Hl] = q_lat
            qf = torch.zeros(T, H, self.qdim, dtype=q.dtype, device=self.device)
            qf[:, h0:h0 + Hl] = q3
            q_lat, q = ql, qf.view(T, H * self.qdim)
        q_lat = q_lat.contiguous()
        if inp.decode:
            row_seq = torch.arange(T, dtype=torch.int32, device=self.device)
        else:
            rows = torch.arange(T, dtype=torch.int32, device=self.device)
            row_seq = (torch.searchsorted(inp.q_start[1:].contiguous(), rows, right=True)).to(torch.int32)
        row_len = (inp.pos + 1).to(torch.int32)
        splits = max(1, min(32, math.ceil(2 * 148 / T)))
        o_lat = ops.mla_attention(q_lat, q, self.qdim, cfg.qk_nope_dim, self.kv[li], inp.block_tables, row_seq,
                                  row_len, H, splits, self.scale)
        o = self._per_head(L.uv, o_lat[:, h0:h0 + Hl], cfg.v_head_dim).reshape(T, Hl * cfg.v_head_dim)
        if T <= GEMV_MAX_T:
            oq = ops.quantize_q8(o, self.x2)
            self._row_parallel(0, lambda m, out: self._lin_q8(L.wo, oq, T, m, out=out), x)
        else:
            ob = o.to(self.act_dtype)
            self._row_parallel(0, lambda m, out: self._lin_bf16(L.wo, ob, T, m, out=out), x)

    def forward(self, inp: StepInput) -> torch.Tensor:
        cfg = self.cfg
        T = inp.ids.numel()
        ops.set_pdl(T <= GEMV_MAX_T)
        x = apply_embed_overrides(ops.embed(self.embed_w, inp.ids), inp)
        for li, L in enumerate(self.layers):
            self._mla(L, li, x, inp, T)
            hb, hq = self._norm(x, L.ffn_norm, T)
            if L.moe is not None:
                self._moe_out(L, hq, hb, T, x)
            else:
                self._row_parallel(1, lambda m, out: self._dense_ffn(L, hq, hb, T, m, out), x)
        xl = x.index_select(0, inp.last_idx) if not inp.decode else x
        _, oq = ops.rmsnorm(xl, self.out_norm, cfg.rms_eps, want_q8=True, x2=self.x2)
        return self._gather_logits(self._lin_q8(self.out_w, oq, xl.shape[0], EPI_STORE_F32))
