"""Python wrappers of the sm_100a kernels (``barq_inference_b200._C``).

The extension is built in-tree by ``setup.py build_ext --inplace``.  On a machine with a GPU a
missing or stale extension is an error (``require_ext``): there is no silent PyTorch fallback.
"""
from __future__ import annotations

import os

import torch

from .qweight import NATIVE, W_BF16, QWeight, cat_rows, interleave_gate_up  # noqa: F401

try:
    from .. import _C  # type: ignore
except ImportError as e:  # pragma: no cover - depends on build state
    _C = None
    _IMPORT_ERROR = e
else:
    _IMPORT_ERROR = None

EPI_STORE_F32, EPI_ADD_F32, EPI_STORE_BF16, EPI_SWIGLU_Q8 = 0, 1, 2, 3
EPI_AR_PUSH = 5  # row-parallel GEMV with the tensor-parallel all-reduce fused in (gemv_allreduce)
EPI_RS_PUSH = 6  # row-parallel GEMM with the reduce-scatter fused in (parallel.comm.Comm.sp_gemm_rs)

# Number of kernel launches issued through these wrappers (bench.py reports launches per step).
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


def require_ext():
    if _C is None:
        raise RuntimeError(
            "barq_inference_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"({_IMPORT_ERROR})")
    return _C


class Q8Act:
    """int8 activation rows + (scale, scale*sum) per 32 values — the GEMV input format.

    With ``x2`` a second int8 term holds the quantized residual (x ~= d*q + dl*ql), which brings the
    activation error from ~2^-8 to ~2^-15 of the group max at twice the dp4a work."""

    __slots__ = ("q", "s", "ql", "dl", "T", "K")

    def __init__(self, q, s, T: int, K: int, ql=None, dl=None):
        self.q, self.s, self.ql, self.dl, self.T, self.K = q, s, ql, dl, T, K

    @staticmethod
    def empty(T: int, K: int, device, x2: bool = False) -> "Q8Act":
        q = torch.empty(T, K, dtype=torch.int8, device=device)
        s = torch.empty(T, K // 32, 2, dtype=torch.float32, device=device)
        if not x2:
            return Q8Act(q, s, T, K)
        return Q8Act(q, s, T, K, torch.empty(T, K, dtype=torch.int8, device=device),
                     torch.empty(T, K // 32, 2, dtype=torch.float32, device=device))

    @property
    def x2(self) -> bool:
        return self.ql is not None

    def rows(self, a: int, b: int) -> "Q8Act":
        lo = (self.ql[a:b], self.dl[a:b]) if self.x2 else (None, None)
        return Q8Act(self.q[a:b], self.s[a:b], b - a, self.K, *lo)

    def outs(self):
        return (self.q, self.s, self.ql, self.dl)


def _ins(x):
    return (None, None, None, None) if x is None else (x.q, x.s, x.ql, x.dl)


def _outs(x):
    return (None, None, None, None) if x is None else x.outs()


def quantize_q8(x: torch.Tensor, x2: bool = False) -> Q8Act:
    T, K = x.shape
    out = Q8Act.empty(T, K, x.device, x2)
    require_ext().quantize_q8(x, T, K, x.stride(0), *out.outs())
    _count()
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, add: torch.Tensor | None = None,
            want_bf16: bool = False, want_q8: bool = False, x2: bool = False, act_dtype=torch.bfloat16):
    """x (f32 [T,H], updated in place by ``add``) -> (activation [T,H] in ``act_dtype`` | None, Q8Act | None)."""
    T, H = x.shape
    ob = torch.empty(T, H, dtype=act_dtype, device=x.device) if want_bf16 else None
    oq = Q8Act.empty(T, H, x.device, x2) if want_q8 else None
    require_ext().rmsnorm(x, add, w, eps, ob, *_outs(oq))
    _count()
    return ob, oq


# Streaming GEMV workspace, one per device: f32 partial-sum slots ([WS_ROWS/128 + 256] x 8 x 128, one
# slot per piece of a row tile that several CTAs share) and int [WS_ROWS/128] tile counters, zero
# between calls (the kernel clears what it used).  Allocated on first use --
# before any CUDA-graph capture, since the engine runs eager steps first.
WS_ROWS = 1 << 18
_GEMV_WS: dict = {}
GEMV_STREAM = os.environ.get("BARQ_GEMV_STREAM", "1") != "0"


def _gemv_ws(w: QWeight):
    if not GEMV_STREAM or w.wtype == W_BF16 or w.N > WS_ROWS:
        return None, None
    key = w.device
    ws = _GEMV_WS.get(key)
    if ws is None:
        ws = (torch.zeros((WS_ROWS // 128 + 256) * 8 * 128, dtype=torch.float32, device=w.device),
              torch.zeros(WS_ROWS // 128, dtype=torch.int32, device=w.device))
        _GEMV_WS[key] = ws
    return ws


NORM_MAX_K = 4096


def gemv_can_fuse_norm(w: QWeight, T: int) -> bool:
    """Whether ``gemv(..., norm=...)`` (RMSNorm computed inside the GEMV) applies."""
    return GEMV_STREAM and w.wtype != W_BF16 and T <= 2 and w.K <= NORM_MAX_K and w.N <= WS_ROWS


def gemv(w: QWeight, x: Q8Act | None, T: int, mode: int = EPI_STORE_F32, out: torch.Tensor | None = None,
         xb: torch.Tensor | None = None, bias: torch.Tensor | None = None, out_q: Q8Act | None = None,
         x2: bool = False, norm: tuple | None = None):
    """Decode GEMV for T <= 8 tokens.  Returns ``out`` (allocated if None for store modes).

    Quantized weights go through the streaming kernel (persistent, bulk-copy fed, stream-K);
    dense bf16 weights through the warp-per-row kernel.  ``norm=(h, weight, eps)`` (f32 h [T, K]):
    the activation is int8(rmsnorm(h) * weight), computed inside the kernel (``x`` unused)."""
    C = require_ext()
    dev = w.device
    wa, wc = _gemv_ws(w)
    nh, nw, neps = (norm if norm is not None else (None, None, 0.0))
    if norm is not None and not gemv_can_fuse_norm(w, T):
        raise ValueError("gemv: fused norm needs a quantized weight, T <= 2 and K <= 4096")
    if mode == EPI_SWIGLU_Q8:
        F = w.N // 2
        if out_q is None:
            out_q = Q8Act.empty(T, F, dev, x2)
        C.qgemv(*w.args(), *_ins(x), xb, T, mode, None, out, *out_q.outs(), bias, F, wa, wc, nh, nw, neps, int(x2))
        _count()
        return out_q
    if out is None:
        dt = torch.bfloat16 if mode == EPI_STORE_BF16 else torch.float32
        out = torch.empty(T, w.N, dtype=dt, device=dev)
    ld = out.stride(0)
    f32 = out if out.dtype == torch.float32 else None
    bf = out if out.dtype == torch.bfloat16 else None
    C.qgemv(*w.args(), *_ins(x), xb, T, mode, f32, bf, None, None, None, None, bias, ld, wa, wc, nh, nw, neps,
            int(x2))
    _count()
    return out


def gemv_can_allreduce(w: QWeight, T: int) -> bool:
    """Whether :func:`gemv_allreduce` (all-reduce fused into the streaming GEMV) applies."""
    return GEMV_STREAM and w.wtype != W_BF16 and T <= 8 and w.N % 128 == 0 and w.N <= WS_ROWS


def gemv_allreduce(w: QWeight, x: Q8Act, T: int, out: torch.Tensor, push, j: int, bias=None) -> torch.Tensor:
    """out (f32 [T, N], the replicated residual) += sum over tensor-parallel ranks of W_r x_r, in
    one kernel: tiles are pushed to every rank over NVLink as they finish.  ``push``: the
    communicator's fused-push state (``Comm.push_args``: int64 device table of the ranks' receive
    buffers for call site j, epoch and counter tensors, rank, wait limit, fault-injection flag)."""
    if not gemv_can_allreduce(w, T):
        raise ValueError("gemv_allreduce: needs a quantized weight, T <= 8 and N % 128 == 0")
    wa, wc = _gemv_ws(w)
    bufs, epoch, done, rank, wait_s, skip = push(j, T, w.N)
    require_ext().qgemv_ar(*w.args(), *_ins(x), T, bias, wa, wc, out, bufs, epoch, done, j, rank, wait_s, int(skip))
    _count()
    return out


def gemm(w: QWeight, x: torch.Tensor, mode: int = EPI_STORE_F32, out: torch.Tensor | None = None,
         bias: torch.Tensor | None = None, k_splits: int = 0) -> torch.Tensor:
    """tcgen05 quantized GEMM: x fp16/bf16 [T, K] -> out (f32 or x.dtype [T, N]; SwiGLU: x.dtype [T, N/2]).

    ``k_splits`` 0 = automatic split-K for the f32 modes (partial tiles summed in split order by the
    last split to finish, so results are deterministic)."""
    T = x.shape[0]
    if mode == EPI_SWIGLU_Q8:
        if out is None:
            out = torch.empty(T, w.N // 2, dtype=x.dtype, device=x.device)
    elif out is None:
        out = torch.empty(T, w.N, dtype=x.dtype if mode == EPI_STORE_BF16 else torch.float32, device=x.device)
    f32 = out if out.dtype == torch.float32 else None
    bf = out if out.dtype != torch.float32 else None
    require_ext().qgemm(*w.args(), x, T, mode, f32, bf, bias, out.stride(0), k_splits)
    _count()
    return out


def set_pdl(on: bool) -> None:
    """Launch the following kernels with (True) or without programmatic dependent launch."""
    require_ext().set_pdl_mode(1 if on else 0)


def gemm_error() -> int:
    """Sticky device error word of the tcgen05 kernels (0 = ok; 0x100|site = bounded wait expired)."""
    return int(require_ext().gemm_error())


def swiglu(gu: torch.Tensor, F: int, want_bf16: bool = True, want_q8: bool = False, x2: bool = False,
           act_dtype=torch.bfloat16):
    T = gu.shape[0]
    ob = torch.empty(T, F, dtype=act_dtype, device=gu.device) if want_bf16 else None
    oq = Q8Act.empty(T, F, gu.device, x2) if want_q8 else None
    require_ext().swiglu(gu, T, F, gu.stride(0), ob, *_outs(oq))
    _count()
    return ob, oq


def rope_kv_write(qkv, pos, slots, cos_t, sin_t, H, Hkv, D, rot, neox, kcache, vcache,
                  q_norm=None, k_norm=None, norm_eps=1e-6, kv_scales=None):
    """RoPE of q / k and the K/V cache write.  ``kv_scales`` (fp8 cache): f32 ``(kscale, vscale)``
    [num_blocks, Hkv, block_size] -- each row is stored as e4m3(x / s) with s = max|x| / 448."""
    T = qkv.shape[0]
    ks, vs = kv_scales if kv_scales is not None else (None, None)
    q_out = torch.empty(T, H, D, dtype=torch.bfloat16, device=qkv.device)
    require_ext().rope_kv_write(qkv, qkv.stride(0), pos, slots, cos_t, sin_t, q_norm, k_norm, norm_eps,
                                T, H, Hkv, D, rot, neox, q_out, kcache, vcache, ks, vs)
    _count()
    return q_out


def decode_splits(B: int, Hkv: int, n_sm: int = 148) -> int:
    """KV splits per (sequence, KV head): just enough CTAs to give every SM one (at most 16).  Each
    decode-attention CTA streams its pages through a deep shared-memory ring, so longer page ranges
    per CTA beat more CTAs: measured on B200 at 32 sequences x 1024 tokens x 8 KV heads, 1 split
    (256 CTAs) runs 39.6 us, 3 splits 44.3 us, 16 splits 76.4 us."""
    return max(1, min(16, -(-n_sm // max(1, B * Hkv))))


def decode_attention(q, kcache, vcache, block_tables, seq_lens, H, Hkv, D, scale, window=0, splits=None,
                     want_q8=True, scratch=None, x2=False, act_dtype=torch.bfloat16, kv_scales=None):
    B = q.shape[0]
    C = require_ext()
    if splits is None:
        splits = decode_splits(B, Hkv)
    if scratch is None:
        scratch = torch.empty(C.decode_attention_scratch_floats(B, H, Hkv, D, splits), dtype=torch.float32,
                              device=q.device)
    out = torch.empty(B, H * D, dtype=act_dtype, device=q.device)
    oq = Q8Act.empty(B, H * D, q.device, x2) if want_q8 else None
    cnt = _attn_counters(q.device, B * Hkv)
    C.decode_attention(q, kcache, vcache, block_tables, seq_lens, B, H, Hkv, D, scale, window, splits, scratch,
                       out, *_outs(oq), cnt, *(kv_scales if kv_scales is not None else (None, None)))
    _count(1 if cnt is not None else 2)
    return out, oq


# Split-merge arrival counters of decode attention, one zeroed int per (sequence, KV head), per
# device; the kernel resets what it used.  Allocated on first use, before any CUDA-graph capture.
_ATTN_CNT: dict = {}
ATTN_FUSED_MERGE = os.environ.get("BARQ_ATTN_MERGE_KERNEL", "0") == "0"


def _attn_counters(device, n: int):
    if not ATTN_FUSED_MERGE:
        return None
    c = _ATTN_CNT.get(device)
    if c is None or c.numel() < n:
        c = torch.zeros(max(n, 4096), dtype=torch.int32, device=device)
        _ATTN_CNT[device] = c
    return c


def prefill_attention(q, kcache, vcache, block_tables, q_start, ctx_lens, max_q, H, Hkv, D, scale, window=0,
                      act_dtype=torch.bfloat16, kv_scales=None, impl: int | None = None):
    """K9 causal varlen prefill attention over the paged cache: returns [T, H * D] in ``act_dtype``.

    ``impl`` 0 runs the mma.sync kernel (``attn_prefill.cu``), 1 the tcgen05 / TMEM / TMA kernel
    (``attn_prefill_tc.cu``; fp16 / bf16 caches with D = 64 or 128, other cases fall back to 0);
    by default ``BARQ_PREFILL_TC`` picks (unset: 0)."""
    if impl is None:
        impl = int(os.environ.get("BARQ_PREFILL_TC", "0"))
    T = q.shape[0]
    S = block_tables.shape[0]
    out = torch.empty(T, H * D, dtype=act_dtype, device=q.device)
    require_ext().prefill_attention(q, kcache, vcache, block_tables, q_start, ctx_lens, S, max_q, H, Hkv, D,
                                    scale, window, out, *(kv_scales if kv_scales is not None else (None, None)),
                                    int(impl))
    _count()
    return out


def mla_kv_write(kv_a: torch.Tensor, norm_w: torch.Tensor, eps: float, cos: torch.Tensor, sin: torch.Tensor,
                 neox: bool, pos: torch.Tensor, slots: torch.Tensor, cache: torch.Tensor, q: torch.Tensor, H: int,
                 qdim: int, rope_off: int) -> None:
    """MLA: latent rows (rmsnorm(c) | rope(k_pe)) into the paged cache; q's rope part rotated in place."""
    require_ext().mla_kv_write(kv_a.contiguous(), norm_w, eps, cos, sin, int(neox), pos, slots, cache, q, H, qdim,
                               rope_off)
    _count()


def mla_attention(q_lat: torch.Tensor, q: torch.Tensor, qdim: int, rope_off: int, cache: torch.Tensor,
                  block_tables: torch.Tensor, row_seq: torch.Tensor, row_len: torch.Tensor, H: int, splits: int,
                  scale: float, impl: int | None = None) -> torch.Tensor:
    """Absorbed MLA attention (K10): returns o_lat f32 [rows, H, 512].

    ``impl`` 0 runs the CUDA-core kernel, 1 the tensor-core kernel (``mla_attn_mma_kernel``); by
    default ``BARQ_MLA_MMA`` picks (unset: 0)."""
    C = require_ext()
    if impl is None:
        impl = int(os.environ.get("BARQ_MLA_MMA", "0"))
    rows = q_lat.shape[0]
    scratch = torch.empty(C.mla_attn_scratch_floats(rows, splits), dtype=torch.float32, device=q_lat.device)
    o = torch.empty(rows, H, 512, dtype=torch.float32, device=q_lat.device)
    C.mla_attention(q_lat, q, qdim, rope_off, cache, block_tables, row_seq, row_len, H, splits, scale, scratch, o,
                    int(impl))
    _count(2)
    return o


EPI_MOE_COMBINE = 4


class MoeRouting:
    """Device buffers of one MoE routing call for up to ``T`` tokens, ``E`` experts, top-``k``."""

    def __init__(self, T: int, E: int, k: int, H: int, dtype, device):
        i32 = dict(dtype=torch.int32, device=device)
        self.T, self.E, self.k = T, E, k
        self.ids = torch.empty(T, k, **i32)
        self.weights = torch.empty(T, k, dtype=torch.float32, device=device)
        self.counts = torch.zeros(E, **i32)  # left zero by the kernels
        self.cursor = torch.empty(E, **i32)
        self.off = torch.empty(E + 1, **i32)
        self.row_tok = torch.empty(T * k, **i32)
        self.row_w = torch.empty(T * k, dtype=torch.float32, device=device)
        self.tok_row = torch.empty(T * k, **i32)
        self.xs = torch.empty(T * k, H, dtype=dtype, device=device)


def moe_router_logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """Router logits f32 [T, E] = x [T, H] (fp16 / bf16) . w [E, H]^T (f32) on the device kernel
    (``moe_router_kernel``); replaces ``x.float() @ w.T`` when ``BARQ_MOE_ROUTER=1``."""
    out = torch.empty(x.shape[0], w.shape[0], dtype=torch.float32, device=x.device)
    require_ext().moe_router_logits(x, w, out)
    _count()
    return out


def router_logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """MoE router logits: the device kernel with ``BARQ_MOE_ROUTER=1`` (opt-in until it has run on a
    GPU), else the f32 library matmul."""
    if os.environ.get("BARQ_MOE_ROUTER") == "1" and w.shape[1] % 4 == 0:
        return moe_router_logits(x, w)
    return x.float() @ w.T


def moe_route(logits: torch.Tensor, x: torch.Tensor, k: int, r: MoeRouting, sigmoid: bool = False,
              renorm: bool = True, n_group: int = 1, topk_group: int = 1, ser_threshold: float = 0.0,
              scale: float = 1.0) -> MoeRouting:
    """Gate + top-k + SER + dispatch of x's rows into expert-major ``r.xs`` (see csrc/kernels/moe.cu)."""
    T = logits.shape[0]
    require_ext().moe_route(logits.contiguous(), k, int(sigmoid), int(renorm), n_group, topk_group, ser_threshold,
                            scale, x.contiguous(), r.ids[:T], r.weights[:T], r.counts, r.cursor, r.off,
                            r.row_tok, r.row_w, r.tok_row, r.xs)
    _count(3)
    return r


def gemm_grouped(w: QWeight, x: torch.Tensor, off: torch.Tensor, n_groups: int, mode: int,
                 out: torch.Tensor | None = None, row_tok=None, row_w=None) -> torch.Tensor:
    """Grouped (per-expert) tcgen05 GEMM over x rows sorted by group (``off`` [n_groups+1] on device).
    SwiGLU mode returns x.dtype [rows, grows/2]; EPI_MOE_COMBINE stores row_w[r] * y[r] into ``out``
    (f32 [rows, grows], indexed by sorted row; :func:`moe_combine` then adds each token's rows)."""
    Tr = x.shape[0]
    grows = w.N // n_groups
    if mode == EPI_SWIGLU_Q8:
        if out is None:
            out = torch.empty(Tr, grows // 2, dtype=x.dtype, device=x.device)
        act, f32, ld = out, None, out.stride(0)
    else:
        if out is None:
            out = torch.empty(Tr, grows, dtype=torch.float32, device=x.device)
        act, f32, ld = None, out, out.stride(0)
    require_ext().qgemm_grouped(*w.args(), x, Tr, mode, f32, act, ld, off, n_groups, grows, row_tok, row_w)
    _count()
    return out


def moe_combine(ys: torch.Tensor, r: "MoeRouting", T: int, lo: torch.Tensor, hi: torch.Tensor,
                x: torch.Tensor) -> torch.Tensor:
    """x[t] += sum over slots j (slot order) of ys[tok_row[t, j]] for rows in [lo, hi) (device int32
    scalars: this rank's window of the expert-sorted rows).  Fixed order: deterministic."""
    require_ext().moe_combine(ys, r.tok_row, lo, hi, T, r.k, x)
    _count()
    return x


def embed(w: QWeight, ids: torch.Tensor) -> torch.Tensor:
    out = torch.empty(ids.numel(), w.K, dtype=torch.float32, device=ids.device)
    require_ext().embed_gather(*w.args(), ids, out)
    _count()
    return out


def dequant_rows(w: QWeight, r0: int = 0, n: int | None = None) -> torch.Tensor:
    n = w.N - r0 if n is None else n
    out = torch.empty(n, w.K, dtype=torch.bfloat16, device=w.device)
    require_ext().dequant_rows(*w.args(), r0, n, out)
    return out


def dequant_dense(w: QWeight, out: torch.Tensor | None = None, dtype=torch.float16) -> torch.Tensor:
    """Whole quantized weight -> row-major ``dtype`` [N, K] (fp16 / bf16), one CTA per weight chunk."""
    if out is None:
        out = torch.empty(w.N, w.K, dtype=dtype, device=w.device)
    require_ext().dequant_dense(*w.args(), out)
    _count()
    return out


def sample(logits, temperature, top_k, top_p, min_p, seeds, steps, allow_mask=None, penalties=None,
           history=None, want_logprob=False):
    B, V = logits.shape
    ids = torch.empty(B, dtype=torch.int32, device=logits.device)
    lp = torch.empty(B, dtype=torch.float32, device=logits.device) if want_logprob else None
    require_ext().sample(logits, B, V, temperature, top_k, top_p, min_p, seeds, steps, ids, lp, allow_mask,
                         penalties, history)
    _count()
    return ids, lp
