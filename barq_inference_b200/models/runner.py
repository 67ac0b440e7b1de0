"""Device model runner: the llama-family decoder (Llama 2/3, Mistral, Mixtral, Qwen2/3) on the
sm_100a kernels, over a paged KV cache.

Parity: ``LlamaTransformer::forward`` (``models/src/transformer.rs:81-498``) — embedding gather,
per layer {RMSNorm, Q/K/V (+bias), RoPE, KV append, causal GQA attention, O proj, residual,
RMSNorm, SwiGLU FFN, residual}, final norm, last-token logits.  Here every step is a fused kernel:

* decode (<= 8 tokens per GEMV launch): RMSNorm -> int8 q8 activations -> dp4a GEMV (K1) with the
  fused QKV projection; RoPE + paged-KV write (K11); paged flash-decode (K8) whose epilogue emits the
  q8 input of the O projection; O/down projections add straight into the f32 residual stream; the
  gate/up GEMV's epilogue computes SiLU(g)*u and its q8 quantization (interleaved gate/up rows).
* prefill: the same graph with the tcgen05 GEMM (K2) for projections and the paged prefill
  attention (K9).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from ..ops import EPI_ADD_F32, EPI_STORE_BF16, EPI_STORE_F32, EPI_SWIGLU_Q8, Q8Act, QWeight
from .config import ModelConfig
from .rope import attn_scale, rope_cos_sin
from .weights import PackedTensor

GEMV_MAX_T = 8
# Optional large-T route (env BARQ_DENSE_T = token threshold, 0 = off, the default): a projection
# dequantizes its whole weight once (csrc dequant_dense) and runs a dense GEMM (a plain library GEMM).
# Measured on Llama-3-8B prefill (8192-token chunks) it was slower than the fused-dequant tcgen05 GEMM
# (33k vs 43k tokens/s: the separate SwiGLU / fp16 output passes cost more than the mainloop saves).
DENSE_T = int(__import__("os").environ.get("BARQ_DENSE_T", "0"))


@dataclass
class StepInput:
    """Device tensors describing one forward step over a batch of sequences."""

    ids: torch.Tensor          # int32 [T]
    pos: torch.Tensor          # int32 [T]
    slots: torch.Tensor        # int64 [T]
    block_tables: torch.Tensor  # int32 [S, max_blocks]
    seq_lens: torch.Tensor     # int32 [S] context length after this step
    last_idx: torch.Tensor     # int64 [S] row of each sequence's last new token
    decode: bool               # every sequence has exactly one new token (T == S)
    q_start: torch.Tensor | None = None  # int32 [S+1] (prefill)
    max_q: int = 1
    # input-embedding overrides (multimodal prompts): rows of the step whose embedding is given
    embed_rows: torch.Tensor | None = None  # int64 [n]
    embed_vals: torch.Tensor | None = None  # f32 [n, hidden]
    # embeddings: when set (f32 [T, hidden]), the final residual stream of every row is copied here
    # before the output norm and head
    hidden_out: torch.Tensor | None = None


def apply_embed_overrides(x: torch.Tensor, inp: StepInput) -> torch.Tensor:
    """Replace the token embeddings of ``inp.embed_rows`` by ``inp.embed_vals`` (image patches)."""
    if inp.embed_rows is not None and inp.embed_rows.numel():
        x.index_copy_(0, inp.embed_rows, inp.embed_vals.to(x.dtype))
    return x


def _qw(pt: PackedTensor, device) -> QWeight:
    N = pt.rows
    return QWeight.from_packed(pt.data, pt.ggml_type, N, pt.cols, device)


def _f32(pt: PackedTensor, device) -> torch.Tensor:
    from .reference import dequant_tensor

    return dequant_tensor(pt).reshape(-1).to(device, torch.float32).contiguous()


class Layer:
    pass


class LlamaRunner:
    def __init__(self, cfg: ModelConfig, tensors: dict[str, PackedTensor], device="cuda",
                 kv_dtype: torch.dtype = torch.float16, use_gemm: bool | None = None, act_x2: bool = True,
                 tp=None, comm=None, pp=None):
        self.cfg = cfg
        # pipeline parallel: ``pp`` (parallel.pp.PPInfo) -- this rank runs layers [l0, l1); stage 0
        # embeds, the last stage computes the logits and broadcasts them
        self.pp = pp
        # tensor parallel: ``tp`` (parallel.tp.TPInfo) describes this rank's shard, ``comm``
        # (parallel.comm.Comm) completes the row-parallel partial sums; None = one GPU
        self.tp, self.comm = tp, comm
        self.device = torch.device(device)
        self.kv_dtype = kv_dtype
        self.scale = attn_scale(cfg)
        self.use_gemm = use_gemm
        # two-term int8 decode activations (accurate mode); False = single int8 term (fastest)
        self.x2 = act_x2
        # dtype of the tensor-core GEMM activations: fp16 (more mantissa, 1-instruction nibble
        # expansion in the GEMM mainloop) unless the family is known to overflow fp16 (DeepSeek)
        self.act_dtype = torch.bfloat16 if cfg.arch.startswith("deepseek") else torch.float16
        dev = self.device
        self.embed_w = _qw(tensors["token_embd.weight"], dev) if "token_embd.weight" in tensors else None
        self.out_norm = _f32(tensors["output_norm.weight"], dev) if "output_norm.weight" in tensors else None
        self.out_w = _qw(tensors["output.weight"], dev) if "output.weight" in tensors else self.embed_w
        self.layers: list[Layer] = []
        F = cfg.ffn
        l0, l1 = (pp.l0, pp.l1) if pp is not None else (0, cfg.n_layers)
        for i in range(l0, l1):
            p = f"blk.{i}."
            L = Layer()
            L.attn_norm = _f32(tensors[p + "attn_norm.weight"], dev)
            L.ffn_norm = _f32(tensors[p + "ffn_norm.weight"], dev)
            q, k, v = (_qw(tensors[p + n], dev) for n in ("attn_q.weight", "attn_k.weight", "attn_v.weight"))
            L.qkv_fused = q.wtype == k.wtype == v.wtype
            L.qkv = ops.cat_rows([q, k, v]) if L.qkv_fused else (q, k, v)
            if cfg.qkv_bias:
                L.qkv_bias = torch.cat([_f32(tensors[p + f"attn_{n}.bias"], dev) for n in "qkv"])
            else:
                L.qkv_bias = None
            L.q_norm = _f32(tensors[p + "attn_q_norm.weight"], dev) if cfg.qk_norm else None
            L.k_norm = _f32(tensors[p + "attn_k_norm.weight"], dev) if cfg.qk_norm else None
            L.wo = _qw(tensors[p + "attn_output.weight"], dev)
            if cfg.layer_is_moe(i):
                from .moe import MoEBlock

                L.moe = MoEBlock(cfg, tensors, p, dev, expert0=tp.expert0 if tp is not None else 0)
            else:
                L.moe = None
                g, u = _qw(tensors[p + "ffn_gate.weight"], dev), _qw(tensors[p + "ffn_up.weight"], dev)
                L.gu_interleaved = g.wtype == u.wtype and g.wtype != ops.W_BF16 and F % 32 == 0
                L.gate_up = ops.interleave_gate_up(g, u) if L.gu_interleaved else (
                    ops.cat_rows([g, u]) if g.wtype == u.wtype else (g, u))
                L.down = _qw(tensors[p + "ffn_down.weight"], dev)
            self.layers.append(L)
        self.cos, self.sin = rope_cos_sin(cfg, cfg.max_ctx, dev)
        if cfg.is_moe:
            from .moe_stats import enable, enabled_by_env

            if enabled_by_env():  # BARQ_MOE_STATS=1: per-expert routed-row counters on the device
                enable(self, dev)

    # ------------------------------------------------------------------ KV cache
    def allocate_kv(self, num_blocks: int, block_size: int = 16) -> list[tuple[torch.Tensor, torch.Tensor]]:
        cfg = self.cfg
        nl = len(self.layers)  # this rank's layers (all of them unless pipeline parallel)
        shape = (nl, 2, num_blocks, cfg.n_kv_heads, block_size, cfg.head_dim)
        kv = torch.zeros(shape, dtype=self.kv_dtype, device=self.device)
        self.kv_storage = kv
        self.kv = [(kv[i, 0], kv[i, 1]) for i in range(nl)]
        # fp8 cache: one f32 scale per stored row (K and V), [layer][2][block][kv head][slot]
        self.kv_scale_storage = None
        self.kv_scales = [None] * nl
        if self.kv_dtype == torch.float8_e4m3fn:
            sc = torch.ones(shape[:-1], dtype=torch.float32, device=self.device)
            self.kv_scale_storage = sc
            self.kv_scales = [(sc[i, 0], sc[i, 1]) for i in range(nl)]
        return self.kv

    def kv_bytes_per_block(self, block_size: int = 16) -> int:
        cfg = self.cfg
        return len(self.layers) * 2 * cfg.n_kv_heads * block_size * cfg.head_dim * torch.finfo(self.kv_dtype).bits // 8

    # ------------------------------------------------------------------ linear layers
    def _lin_q8(self, w, x: Q8Act, T: int, mode: int, out=None, bias=None, xb=None):
        """GEMV in launches of <= 8 tokens."""
        if isinstance(w, tuple):
            outs = [self._lin_q8(wi, x, T, EPI_STORE_F32, xb=xb) for wi in w]
            r = torch.cat(outs, 1)
            if bias is not None:
                r += bias
            if mode == EPI_ADD_F32:
                out += r
                return out
            return r
        if mode == EPI_SWIGLU_Q8:
            oq = Q8Act.empty(T, w.N // 2, self.device, self.x2)
            for t0 in range(0, T, GEMV_MAX_T):
                t1 = min(T, t0 + GEMV_MAX_T)
                ops.gemv(w, x.rows(t0, t1) if x is not None else None, t1 - t0, mode, out_q=oq.rows(t0, t1),
                         xb=None if xb is None else xb[t0:t1])
            return oq
        if out is None:
            out = torch.empty(T, w.N, dtype=torch.bfloat16 if mode == EPI_STORE_BF16 else torch.float32,
                              device=self.device)
        for t0 in range(0, T, GEMV_MAX_T):
            t1 = min(T, t0 + GEMV_MAX_T)
            ops.gemv(w, x.rows(t0, t1) if x is not None else None, t1 - t0, mode, out=out[t0:t1], bias=bias,
                     xb=None if xb is None else xb[t0:t1].contiguous())
        return out

    def _row_parallel(self, j: int, fn, x: torch.Tensor, gemv=None) -> None:
        """Add a row-parallel layer's output into the residual ``x``.  ``fn(mode, out)`` writes this
        rank's partial with EPI_ADD_F32 (into x) or EPI_STORE_F32 (into a buffer).  One GPU: plain
        add.  Fused TP (decode-sized messages): store into the symmetric buffer j, then one kernel adds
        every rank's partial.  NCCL TP (and large messages): rank 0 adds into x, the others store
        into x, then an all-reduce.  ``gemv=(w, act, bias)``: the layer is one streaming GEMV, so with
        the fused communicator its all-reduce runs inside that GEMV (``ops.gemv_allreduce``)."""
        c = self.comm
        if c is None or c.world == 1:
            fn(EPI_ADD_F32, x)
        elif (c.fused and gemv is not None and not isinstance(gemv[0], tuple) and x.shape[0] <= GEMV_MAX_T
              and c.push_ok(x.shape[0], x.shape[1]) and ops.gemv_can_allreduce(gemv[0], x.shape[0])):
            ops.gemv_allreduce(gemv[0], gemv[1], x.shape[0], x, c.push_args, j, bias=gemv[2])
        elif c.fused and x.numel() <= c.fused_max_elems:  # large (prefill) messages go through NCCL
            fn(EPI_STORE_F32, c.partial(j, x.shape[0], x.shape[1]))
            c.allreduce_add(j, x)
        else:
            fn(EPI_ADD_F32 if c.rank == 0 else EPI_STORE_F32, x)
            c.all_reduce(x)

    def _moe_out(self, L, hq, hb, T, x) -> None:
        def fn(mode, out):
            if mode == EPI_STORE_F32:
                out.zero_()
            L.moe.forward(self, hq, hb, T, out)
        self._row_parallel(1, fn, x)

    # ------------------------------------------------------------------ pipeline stages
    def _stage_input(self, inp: StepInput) -> torch.Tensor:
        """Stage 0 (or a single GPU): embeddings.  Later stages: the previous stage's hidden states."""
        if self.pp is None or self.pp.stage == 0:
            return apply_embed_overrides(ops.embed(self.embed_w, inp.ids), inp)
        x = torch.empty(inp.ids.numel(), self.cfg.hidden, dtype=torch.float32, device=self.device)
        self.pp.recv(x)
        return x

    def _stage_forward(self, x: torch.Tensor, inp: StepInput) -> bool:
        """True if this stage hands its hidden states on (and computes no logits)."""
        if self.pp is None or self.pp.is_last:
            return False
        self.pp.send(x)
        return True

    def _stage_logits(self, inp: StepInput, logits: torch.Tensor | None = None) -> torch.Tensor:
        """Every stage returns the same logits: the last stage broadcasts them."""
        if self.pp is None:
            return logits
        if logits is None:
            logits = torch.empty(inp.last_idx.numel(), self.cfg.vocab, dtype=torch.float32, device=self.device)
        self.pp.broadcast_logits(logits)
        return logits

    def _gather_logits(self, logits: torch.Tensor) -> torch.Tensor:
        """Vocab-parallel head: every rank holds a slice of the vocabulary; all-gather the logits."""
        if self.comm is not None and self.comm.world > 1 and self.tp is not None and self.tp.vocab_local:
            logits = self.comm.all_gather_cols(logits)
        return logits

    def _head(self, x_last: torch.Tensor) -> torch.Tensor:
        return self._gather_logits(self._norm_lin(self.out_w, x_last, self.out_norm, x_last.shape[0], EPI_STORE_F32))

    def _norm_lin(self, w, x: torch.Tensor, norm_w: torch.Tensor, T: int, mode: int, out=None, bias=None):
        """RMSNorm(x) -> int8 -> GEMV.  For 1-2 tokens on a quantized weight the norm runs inside the
        streaming GEMV (no separate launch); otherwise RMSNorm then ``_lin_q8``."""
        eps = self.cfg.rms_eps
        if isinstance(w, QWeight) and ops.gemv_can_fuse_norm(w, T):
            if mode == EPI_SWIGLU_Q8:
                oq = Q8Act.empty(T, w.N // 2, self.device, self.x2)
                ops.gemv(w, None, T, mode, out_q=oq, x2=self.x2, norm=(x, norm_w, eps))
                return oq
            if out is None:
                out = torch.empty(T, w.N, dtype=torch.float32, device=self.device)
            ops.gemv(w, None, T, mode, out=out, bias=bias, x2=self.x2, norm=(x, norm_w, eps))
            return out
        hb, hq = ops.rmsnorm(x, norm_w, eps, want_q8=True, want_bf16=self._needs_bf16(w), x2=self.x2)
        return self._lin_q8(w, hq, T, mode, out=out, bias=bias, xb=hb)

    def _dense_ok(self, w, T: int) -> bool:
        return DENSE_T > 0 and T >= DENSE_T and isinstance(w, QWeight) and w.wtype != ops.W_BF16

    def _dense_gemm(self, w, xb: torch.Tensor, mode: int, out=None, bias=None):
        """Large-T projection: dequantize w into a reused scratch, then a dense GEMM."""
        n = w.N * w.K
        sc = getattr(self, "_dense_scratch", None)
        if sc is None or sc.numel() < n or sc.dtype != xb.dtype:
            sc = self._dense_scratch = torch.empty(n, dtype=xb.dtype, device=self.device)
        wd = ops.dequant_dense(w, sc[:n].view(w.N, w.K))
        y = torch.matmul(xb, wd.t())
        if mode == EPI_SWIGLU_Q8:  # rows interleaved [32 gate | 32 up] per group
            T = y.shape[0]
            g4 = y.view(T, -1, 2, 32)
            return (torch.nn.functional.silu(g4[:, :, 0, :].float()) * g4[:, :, 1, :].float()).reshape(T, -1).to(
                xb.dtype)
        if bias is not None:
            y = y.float() + bias
        if mode == EPI_ADD_F32:
            out.add_(y)
            return out
        if out is None:
            return y.float()
        out.copy_(y)
        return out

    def _lin_bf16(self, w, xb: torch.Tensor, T: int, mode: int, out=None, bias=None):
        """Projection of bf16 activations [T, K] on the tcgen05 GEMM (K2)."""
        if self._dense_ok(w, T):
            return self._dense_gemm(w, xb, mode, out=out, bias=bias)
        if isinstance(w, tuple):
            r = torch.cat([self._lin_bf16(wi, xb, T, EPI_STORE_F32) for wi in w], 1)
            if bias is not None:
                r += bias
            if mode == EPI_ADD_F32:
                out += r
                return out
            return r
        if w.wtype == ops.W_BF16:  # dense weights (non-blocked GGUF tensors): GEMV in chunks
            xb = xb.to(torch.bfloat16)
            if out is None:
                out = torch.empty(T, w.N, dtype=torch.float32, device=self.device)
            for t0 in range(0, T, GEMV_MAX_T):
                t1 = min(T, t0 + GEMV_MAX_T)
                ops.gemv(w, None, t1 - t0, mode, out=out[t0:t1], bias=bias, xb=xb[t0:t1].contiguous())
            return out
        return ops.gemm(w, xb, mode, out=out, bias=bias)

    def _needs_bf16(self, w) -> bool:
        if isinstance(w, tuple):
            return any(self._needs_bf16(x) for x in w)
        return w.wtype == ops.W_BF16

    # ------------------------------------------------------------------ forward
    def forward(self, inp: StepInput) -> torch.Tensor:
        """Logits (f32) of the last new token of each sequence: [S, vocab]."""
        T = inp.ids.numel()
        # programmatic dependent launch pays off where launches are short (GEMV-sized steps); next to
        # the persistent GEMM, early-launched waiting CTAs only take SM resources
        ops.set_pdl(T <= GEMV_MAX_T)
        if T > GEMV_MAX_T and self.use_gemm is not False:
            return self._forward_gemm(inp)
        return self._forward_gemv(inp)

    def _attention(self, L, li, qkv, inp, T, want_q8):
        cfg = self.cfg
        H, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        kc, vc = self.kv[li]
        ks = self.kv_scales[li]
        q = ops.rope_kv_write(qkv, inp.pos, inp.slots, self.cos, self.sin, H, Hkv, D, cfg.rot_dim,
                              cfg.rope_neox, kc, vc, L.q_norm, L.k_norm, cfg.rms_eps, kv_scales=ks)
        if inp.decode:
            return ops.decode_attention(q, kc, vc, inp.block_tables, inp.seq_lens, H, Hkv, D, self.scale,
                                        cfg.sliding_window, want_q8=want_q8, x2=self.x2, act_dtype=self.act_dtype,
                                        kv_scales=ks)
        ab = ops.prefill_attention(q, kc, vc, inp.block_tables, inp.q_start, inp.seq_lens, inp.max_q,
                                   H, Hkv, D, self.scale, cfg.sliding_window, act_dtype=self.act_dtype,
                                   kv_scales=ks)
        return ab, (ops.quantize_q8(ab, self.x2) if want_q8 else None)

    def _sp_ok(self, T: int) -> bool:
        """Whether this step runs sequence-parallel with the collectives fused into the GEMMs
        (tensor parallel over NVLink, every projection a quantized tcgen05 GEMM)."""
        c = self.comm
        if c is None or c.world == 1 or self.pp is not None or not c.sp_ok(T) or c.sp_act_dtype != self.act_dtype:
            return False
        ok = getattr(self, "_sp_layers_ok", None)
        if ok is None:
            q = lambda w: isinstance(w, QWeight) and w.wtype != ops.W_BF16  # noqa: E731
            dense_ok = lambda L: L.gu_interleaved and q(L.gate_up) and q(L.down) and \
                L.down.N == self.cfg.hidden  # noqa: E731
            ok = self._sp_layers_ok = self.embed_w is not None and q(self.out_w) and all(
                (c.ep_ok(L.moe) if L.moe is not None else dense_ok(L)) and q(L.qkv) and q(L.wo)
                and L.wo.N == self.cfg.hidden for L in self.layers)
        return ok

    def _forward_sp(self, inp: StepInput) -> torch.Tensor:
        """Tensor parallel, sequence-parallel residual: this rank keeps token rows [a, b) of the
        residual stream.  Per layer: qkv GEMM on the gathered normalized rows (waiting per token
        tile), attention on this rank's heads, o_proj GEMM whose epilogue reduce-scatters into the
        owners, owner-side residual add + RMSNorm + all-gather, gate|up GEMM, down GEMM with the same
        reduce-scatter, and the next norm.  MoE layers instead send this rank's normalized rows to the
        experts' ranks and gather the weighted outputs back (``Comm.ep_moe``).  No NCCL call and no
        separate all-reduce kernel."""
        cfg, c = self.cfg, self.comm
        T = inp.ids.numel()
        eps = cfg.rms_eps
        chunk, a, b = c.sp_rows(T)
        x = apply_embed_overrides(ops.embed(self.embed_w, inp.ids), inp)[a:b].contiguous()
        c.sp_reduce_norm_ag(1, x, T, self.layers[0].attn_norm, eps, reduce=False)
        for li, L in enumerate(self.layers):
            qkv = c.sp_gemm_ag(L.qkv, 1, T, EPI_STORE_F32, bias=L.qkv_bias)
            ab, _ = self._attention(L, li, qkv, inp, T, want_q8=False)
            c.sp_gemm_rs(L.wo, ab, 0)
            nxt = self.layers[li + 1].attn_norm if li + 1 < len(self.layers) else self.out_norm
            if L.moe is not None:  # expert parallel: this rank's rows go to the experts' ranks and back
                c.sp_reduce_norm_ag(0, x, T, L.ffn_norm, eps, self_only=True)
                c.ep_moe(L.moe, c.sp_ag[0][a:b], x, getattr(self, "ser_threshold", 0.0))
                c.sp_reduce_norm_ag(1, x, T, nxt, eps, reduce=False)
                continue
            c.sp_reduce_norm_ag(0, x, T, L.ffn_norm, eps)
            h = c.sp_gemm_ag(L.gate_up, 0, T, EPI_SWIGLU_Q8)
            c.sp_gemm_rs(L.down, h, 1)
            c.sp_reduce_norm_ag(1, x, T, nxt, eps)
        if inp.hidden_out is not None:  # embeddings: the whole residual stream (rare; NCCL gather)
            import torch.distributed as dist

            pad = torch.zeros(chunk, cfg.hidden, dtype=torch.float32, device=self.device)
            pad[:b - a] = x
            full = torch.empty(chunk * c.world, cfg.hidden, dtype=torch.float32, device=self.device)
            dist.all_gather_into_tensor(full, pad, group=c.group)
            inp.hidden_out.copy_(full[:T])
        ob = c.sp_gathered(1, T)  # out_norm(x) of every row
        xl = ob.index_select(0, inp.last_idx) if not inp.decode else ob
        S = xl.shape[0]
        if S <= GEMV_MAX_T:
            xq = ops.quantize_q8(xl.float(), self.x2)
            logits = self._lin_q8(self.out_w, xq, S, EPI_STORE_F32, xb=xl.to(torch.bfloat16))
        else:
            logits = self._lin_bf16(self.out_w, xl.contiguous(), S, EPI_STORE_F32)
        return self._stage_logits(inp, self._gather_logits(logits))

    def _forward_gemm(self, inp: StepInput) -> torch.Tensor:
        """Many tokens (prefill, batched decode): bf16 activations on the tcgen05 GEMM."""
        cfg = self.cfg
        T = inp.ids.numel()
        if self._sp_ok(T):
            return self._forward_sp(inp)
        x = self._stage_input(inp)
        for li, L in enumerate(self.layers):
            hb, _ = ops.rmsnorm(x, L.attn_norm, cfg.rms_eps, want_bf16=True, act_dtype=self.act_dtype)
            qkv = self._lin_bf16(L.qkv, hb, T, EPI_STORE_F32, bias=L.qkv_bias)
            ab, _ = self._attention(L, li, qkv, inp, T, want_q8=False)
            self._row_parallel(0, lambda m, o: self._lin_bf16(L.wo, ab, T, m, out=o), x)
            hb, hq = ops.rmsnorm(x, L.ffn_norm, cfg.rms_eps, want_bf16=True,
                                 want_q8=L.moe is not None, x2=self.x2, act_dtype=self.act_dtype)
            if L.moe is not None:
                self._moe_out(L, hq, hb, T, x)
                continue
            if L.gu_interleaved and self._dense_ok(L.gate_up, T):
                h = self._dense_gemm(L.gate_up, hb, EPI_SWIGLU_Q8)
            elif L.gu_interleaved:
                h = ops.gemm(L.gate_up, hb, EPI_SWIGLU_Q8)
            else:
                gu = self._lin_bf16(L.gate_up, hb, T, EPI_STORE_F32)
                h, _ = ops.swiglu(gu, cfg.ffn, want_bf16=True, act_dtype=self.act_dtype)
            self._row_parallel(1, lambda m, o: self._lin_bf16(L.down, h, T, m, out=o), x)
        if self._stage_forward(x, inp):
            return self._stage_logits(inp)
        if inp.hidden_out is not None:
            inp.hidden_out.copy_(x)
        xl = x.index_select(0, inp.last_idx) if not inp.decode else x
        ob, oq = ops.rmsnorm(xl, self.out_norm, cfg.rms_eps, want_bf16=True, act_dtype=self.act_dtype)
        if xl.shape[0] <= GEMV_MAX_T:
            _, oq = ops.rmsnorm(xl, self.out_norm, cfg.rms_eps, want_q8=True, x2=self.x2)
            return self._stage_logits(inp, self._gather_logits(
                self._lin_q8(self.out_w, oq, xl.shape[0], EPI_STORE_F32, xb=ob.to(torch.bfloat16))))
        return self._stage_logits(inp, self._gather_logits(self._lin_bf16(self.out_w, ob, xl.shape[0], EPI_STORE_F32)))

    def _forward_gemv(self, inp: StepInput) -> torch.Tensor:
        cfg = self.cfg
        T = inp.ids.numel()
        H, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        x = self._stage_input(inp)
        for li, L in enumerate(self.layers):
            kc, vc = self.kv[li]
            qkv = self._norm_lin(L.qkv, x, L.attn_norm, T, EPI_STORE_F32, bias=L.qkv_bias)
            ks = self.kv_scales[li]
            q = ops.rope_kv_write(qkv, inp.pos, inp.slots, self.cos, self.sin, H, Hkv, D, cfg.rot_dim,
                                  cfg.rope_neox, kc, vc, L.q_norm, L.k_norm, cfg.rms_eps, kv_scales=ks)
            if inp.decode:
                ab, aq = ops.decode_attention(q, kc, vc, inp.block_tables, inp.seq_lens, H, Hkv, D, self.scale,
                                              cfg.sliding_window, x2=self.x2, kv_scales=ks)
            else:
                ab = ops.prefill_attention(q, kc, vc, inp.block_tables, inp.q_start, inp.seq_lens, inp.max_q,
                                           H, Hkv, D, self.scale, cfg.sliding_window, kv_scales=ks)
                aq = ops.quantize_q8(ab, self.x2)
            self._row_parallel(0, lambda m, o: self._lin_q8(L.wo, aq, T, m, out=o, xb=ab), x, gemv=(L.wo, aq, None))
            if L.moe is not None:
                hb, hq = ops.rmsnorm(x, L.ffn_norm, cfg.rms_eps, want_q8=True, want_bf16=True, x2=self.x2)
                self._moe_out(L, hq, hb, T, x)
                continue
            down_bf16 = self._needs_bf16(L.down)
            if L.gu_interleaved and not down_bf16:
                h2 = self._norm_lin(L.gate_up, x, L.ffn_norm, T, EPI_SWIGLU_Q8)
                self._row_parallel(1, lambda m, o: self._lin_q8(L.down, h2, T, m, out=o), x, gemv=(L.down, h2, None))
            else:
                hb, hq = ops.rmsnorm(x, L.ffn_norm, cfg.rms_eps, want_q8=True,
                                     want_bf16=self._needs_bf16(L.gate_up), x2=self.x2)
                gu = self._lin_q8(L.gate_up, hq, T, EPI_STORE_F32, xb=hb)
                if L.gu_interleaved:  # undo the 32-row interleave for the elementwise kernel
                    gu = gu.view(T, -1, 2, 32).transpose(1, 2).reshape(T, -1).contiguous()
                hb2, hq2 = ops.swiglu(gu, cfg.ffn, want_bf16=down_bf16, want_q8=cfg.ffn % 32 == 0 and not down_bf16,
                                      x2=self.x2)
                self._row_parallel(1, lambda m, o: self._lin_q8(L.down, hq2, T, m, out=o, xb=hb2), x,
                                   gemv=(L.down, hq2, None) if hq2 is not None else None)
        if self._stage_forward(x, inp):
            return self._stage_logits(inp)
        if inp.hidden_out is not None:
            inp.hidden_out.copy_(x)
        xl = x.index_select(0, inp.last_idx) if not inp.decode else x
        return self._stage_logits(inp, self._head(xl))
