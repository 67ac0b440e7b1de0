"""Communication backend for tensor / expert parallelism: one process per GPU over NCCL.

Parity: ``NcclCommunicator`` / ``MultiGpuManager`` (``backend/src/cuda_multi_gpu.rs:197-233, 400-453``)
and ``CommBackend`` (``advanced/src/tensor_parallel.rs:28-37``), all stubs in the reference.

* Bootstrap: ``torch.distributed`` (NCCL backend) from the usual RANK / WORLD_SIZE / MASTER_* env;
  every collective has the process group's timeout, so a rank that dies makes the others raise
  instead of waiting forever.
* Baseline path: ``all_reduce`` / ``all_gather`` through NCCL.
* Fused path (``fused=True``): a symmetric allocation (every rank maps every peer's buffer over
  NVLink) holds two partial-sum buffers and the barrier flags; row-parallel layers store their
  partial into the local buffer and ``allreduce_add`` (csrc/kernels/allreduce.cu) sums the peers'
  partials into the residual stream in one kernel -- a one-shot all-reduce with the residual add
  fused, no NCCL launch on the decode path.
* Fused GEMV + all-reduce (decode, up to ``push_rows`` tokens): the same allocation also holds two
  receive buffers of ``world`` slots of 64-bit (epoch, value) words; the row-parallel streaming
  GEMV itself stores every finished tile into all peers' slot for this rank and adds the peers'
  tiles as they arrive (``ops.gemv_allreduce``), so the all-reduce costs no launch of its own.
* Sequence-parallel GEMM path (``sp_tokens``, more than 8 tokens: prefill and batched decode): a second
  symmetric allocation holds per-rank receive slots, two gather buffers and their flags.  The
  row-parallel tcgen05 GEMM pushes each output tile into its owner's slots (reduce-scatter fused into
  the GEMM epilogue), the owner's ``sp_reduce_norm_ag`` kernel adds the partials into its rows of the
  residual stream, normalizes them and pushes the rows to every rank (all-gather), and the next
  column-parallel GEMM waits per token tile for those rows (csrc/kernels/tp_fused.cu).
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

from ..ops import require_ext


class Comm:
    def __init__(self, device: torch.device, fused: bool = True, max_elems: int = 0,
                 timeout_s: float = 120.0, wait_s: float = 20.0, hidden: int = 0, push_rows: int = 8, group=None,
                 sp_tokens: int = 0, act_dtype=torch.float16, ep_experts: int = 0, ep_topk: int = 0):
        """``group``: the tensor-parallel process group (None = every rank; a subgroup when tensor
        parallelism is combined with pipeline stages).  ``rank`` / ``world`` are group-local."""
        if not dist.is_initialized():
            dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=timeout_s))
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device
        # device-side barrier limit of the fused all-reduce: ranks may legitimately drift apart by
        # seconds (graph capture, garbage collection); a longer silence is a failed peer
        self.wait_s = wait_s
        self.fused = fused and self.world > 1
        # the one-shot kernel wins on latency-bound (decode) messages; NCCL's ring/NVLS algorithms
        # win on bandwidth-bound ones (prefill), which therefore stay on NCCL
        self.fused_max_elems = 256 * 1024
        self.skip_signal = False  # fault injection (BARQ_FAULT skip_flag)
        self.max_elems = max_elems
        # fused GEMV + all-reduce receive buffers: [2][world][push_rows * hidden] 64-bit words
        self.push_elems = push_rows * hidden if (self.fused and hidden) else 0
        self.push_fused = self.push_elems > 0 and os.environ.get("BARQ_AR_PUSH", "1") != "0"
        if self.fused:
            self._setup_symmetric(max_elems)
        # sequence-parallel buffers: up to sp_tokens rows per step on the fused GEMM path
        self.sp_tokens = sp_tokens if (self.fused and hidden and os.environ.get("BARQ_SP", "1") != "0") else 0
        if self.sp_tokens:
            self._setup_sp(self.sp_tokens, hidden, act_dtype)
        # expert-parallel all-to-all buffers (MoE models on the sequence-parallel path)
        self.ep_experts = ep_experts if (self.sp_tokens and ep_experts and ep_experts % self.world == 0) else 0
        if self.ep_experts:
            self._setup_ep(ep_experts, ep_topk, self.sp_tokens, hidden, act_dtype)

    # ------------------------------------------------------------------ fused path
    def _setup_symmetric(self, n: int) -> None:
        import torch.distributed._symmetric_memory as symm

        n = (n + 63) // 64 * 64
        flag_words = 64 * 8  # kArMaxBlocks x kArMaxRanks u32
        pe = self.push_elems
        self.buf = symm.empty(2 * n + flag_words + 2 * self.world * pe * 2, dtype=torch.float32, device=self.device)
        self.buf.zero_()
        self.hdl = symm.rendezvous(self.buf, self.group if self.group is not None else dist.group.WORLD)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        base = list(self.hdl.buffer_ptrs)
        self._bufs = [[p + j * n * 4 for p in base] for j in (0, 1)]
        self._flags = [p + 2 * n * 4 for p in base]
        self._n = n
        # NVLS (BARQ_AR_MULTIMEM=1): multicast addresses of the two partial buffers, when the
        # allocation is bound to a multicast object; 0 selects the peer-load form
        mc = int(getattr(self.hdl, "multicast_ptr", 0) or 0) if os.environ.get("BARQ_AR_MULTIMEM") == "1" else 0
        self._mc_bufs = [mc + j * n * 4 if mc else 0 for j in (0, 1)]
        self.epoch = torch.zeros(64, dtype=torch.int32, device=self.device)
        off = 2 * n + flag_words  # a multiple of 64 floats: the words are 8-byte aligned
        self._push_bufs = [torch.tensor([p + (off + j * self.world * pe * 2) * 4 for p in base], dtype=torch.int64,
                                        device=self.device) for j in (0, 1)]
        self.push_epoch = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.push_done = torch.zeros(2, dtype=torch.int32, device=self.device)

    def _setup_sp(self, T_max: int, H: int, act_dtype) -> None:
        import torch.distributed._symmetric_memory as symm

        W = self.world
        chunk = -(-T_max // W)
        max_tiles = -(-H // 128) * -(-T_max // 32)
        al = lambda n: (n + 255) // 256 * 256  # noqa: E731  (byte offsets kept 256-aligned)
        o_slots = 0
        o_ag = o_slots + al(W * chunk * H * 4)
        o_rsf = o_ag + 2 * al(T_max * H * 2)
        o_agf = o_rsf + 2 * al(W * max_tiles * 4)
        total = o_agf + 2 * al(T_max * 4)
        self.sp_buf = symm.empty(total, dtype=torch.uint8, device=self.device)
        self.sp_buf.zero_()
        self.sp_hdl = symm.rendezvous(self.sp_buf, self.group if self.group is not None else dist.group.WORLD)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        base = list(self.sp_hdl.buffer_ptrs)
        self.sp_H, self.sp_max_tiles, self.sp_act_dtype = H, max_tiles, act_dtype
        self._sp_slots = [p + o_slots for p in base]
        self._sp_rsf = [[p + o_rsf + j * al(W * max_tiles * 4) for p in base] for j in (0, 1)]
        self._sp_ag = [[p + o_ag + j * al(T_max * H * 2) for p in base] for j in (0, 1)]
        self._sp_agf = [[p + o_agf + j * al(T_max * 4) for p in base] for j in (0, 1)]
        b = self.sp_buf
        self.sp_slots = b[o_slots:o_slots + W * chunk * H * 4].view(torch.float32)
        self.sp_rs_flags = [b[o_rsf + j * al(W * max_tiles * 4):][:W * max_tiles * 4].view(torch.int32) for j in (0, 1)]
        self.sp_ag = [b[o_ag + j * al(T_max * H * 2):][:T_max * H * 2].view(act_dtype).view(T_max, H) for j in (0, 1)]
        self.sp_ag_flags = [b[o_agf + j * al(T_max * 4):][:T_max * 4].view(torch.int32) for j in (0, 1)]
        self.sp_epoch = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.sp_done = torch.zeros(2, dtype=torch.int32, device=self.device)

    def _setup_ep(self, E: int, k: int, T_max: int, H: int, act_dtype) -> None:
        import torch.distributed._symmetric_memory as symm

        W = self.world
        chunk = -(-T_max // W)
        cap = W * chunk * k  # every routed row of every rank could land on one rank
        al = lambda n: (n + 255) // 256 * 256  # noqa: E731
        o_cnt = 0
        o_cf = o_cnt + al(W * E * 4)
        o_df = o_cf + al(W * 4)
        o_yf = o_df + al(W * 4)
        o_rx = o_yf + al(W * 4)
        o_ys = o_rx + al(cap * H * 2)
        total = o_ys + al(cap * H * 4)
        self.ep_buf = symm.empty(total, dtype=torch.uint8, device=self.device)
        self.ep_buf.zero_()
        self.ep_hdl = symm.rendezvous(self.ep_buf, self.group if self.group is not None else dist.group.WORLD)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        base = list(self.ep_hdl.buffer_ptrs)
        self._ep = {n: [p + o for p in base] for n, o in
                    (("cnt", o_cnt), ("cf", o_cf), ("df", o_df), ("yf", o_yf), ("rx", o_rx), ("ys", o_ys))}
        b = self.ep_buf
        self.ep_recv_x = b[o_rx:o_rx + cap * H * 2].view(act_dtype).view(cap, H)
        self.ep_ys = b[o_ys:o_ys + cap * H * 4].view(torch.float32).view(cap, H)
        self.ep_cap, self.ep_topk = cap, k
        i32 = dict(dtype=torch.int32, device=self.device)
        self.ep_epoch = torch.zeros(1, **i32)
        self.ep_done = torch.zeros(2, **i32)
        self.ep_counts = torch.zeros(E, **i32)   # left zero by the dispatch kernel
        self.ep_cursor = torch.zeros(E, **i32)
        self.ep_recv_off = torch.zeros(E // W + 1, **i32)
        self.ep_ids = torch.zeros(chunk, k, **i32)
        self.ep_w = torch.zeros(chunk, k, dtype=torch.float32, device=self.device)
        self.ep_pos = torch.zeros(chunk * k * 2, **i32)
        self._ep_dummy = torch.zeros(max(E + 1, chunk * k), **i32)
        self._ep_dummy_f = torch.zeros(max(E + 1, chunk * k), dtype=torch.float32, device=self.device)

    def ep_ok(self, moe) -> bool:
        return bool(self.ep_experts) and moe.E == self.ep_experts and moe.k == self.ep_topk and \
            moe.E_local * self.world == moe.E and moe.shared is None

    def ep_moe(self, moe, hb: torch.Tensor, x: torch.Tensor, ser: float = 0.0) -> None:
        """Expert-parallel MoE FFN of this rank's token rows: x (f32 [rows, H]) += sum over the routed
        experts of gate_weight * expert(hb), with the rows sent to and gathered from the experts'
        ranks over NVLink (moe.cu ep_* kernels; no NCCL, no replicated routing)."""
        from .. import ops

        C = require_ext()
        rows = hb.shape[0]
        logits = ops.router_logits(hb, moe.router)
        ids, wts, d = self.ep_ids[:rows], self.ep_w[:rows], self._ep_dummy
        ra = moe._route_args(ser)
        C.moe_route(logits.contiguous(), moe.k, int(ra["sigmoid"]), int(ra["renorm"]), ra["n_group"],
                    ra["topk_group"], ra["ser_threshold"], ra["scale"], hb, ids, wts, self.ep_counts, d, d, d, self._ep_dummy_f,
                    d, None)
        ep = self._ep
        args = (self.rank, moe.E, moe.E_local, moe.k, rows, ids, wts, self.ep_counts, self.ep_cursor, ep["cnt"],
                ep["cf"], hb, ep["rx"], ep["df"], self.ep_pos, self.ep_recv_off, ep["ys"], ep["yf"])
        C.ep_call(0, *args, None, self.ep_epoch, self.ep_done, self.ep_cap, self.wait_s)
        h = ops.gemm_grouped(moe.gate_up, self.ep_recv_x, self.ep_recv_off, moe.E_local, ops.EPI_SWIGLU_Q8)
        ops.gemm_grouped(moe.down, h, self.ep_recv_off, moe.E_local, ops.EPI_STORE_F32, out=self.ep_ys)
        C.ep_call(1, *args, x, self.ep_epoch, self.ep_done, self.ep_cap, self.wait_s)
        ops._count(5)

    # ------------------------------------------------------------------ sequence-parallel path
    # Fewest tokens per step that run sequence-parallel.  Below it (batched decode) the partials
    # go through the one-shot all-reduce kernel: at 32 tokens on 2 B200 the per-site reduce kernel
    # and flag round trips of the sequence-parallel path cost more than they save (6.65 vs 5.25 ms
    # per Llama-3-8B step), while prefill gains (76k vs 53k tok/s).
    sp_min_tokens = int(os.environ.get("BARQ_SP_MIN_TOKENS", "128"))

    def sp_ok(self, T: int) -> bool:
        return bool(self.sp_tokens) and max(9, self.sp_min_tokens) <= T <= self.sp_tokens

    def sp_rows(self, T: int) -> tuple[int, int, int]:
        """(chunk, first, end): this rank owns token rows [first, end) of a T-row step."""
        chunk = -(-T // self.world)
        a = min(T, self.rank * chunk)
        return chunk, a, min(T, a + chunk)

    def sp_gemm_rs(self, w, x: torch.Tensor, site: int, bias=None) -> None:
        """Row-parallel GEMM whose epilogue pushes every output tile into its owner's slots."""
        from .. import ops

        T = x.shape[0]
        chunk = -(-T // self.world)
        require_ext().qgemm_sp(*w.args(), x, T, ops.EPI_RS_PUSH, None, None, bias, w.N, self._sp_slots,
                               self._sp_rsf[site], self.sp_epoch[site:site + 1], self.rank, chunk, self.sp_max_tiles,
                               None, None, self.wait_s)
        ops._count()

    def sp_gemm_ag(self, w, site: int, T: int, mode: int, out=None, bias=None) -> torch.Tensor:
        """Column-parallel GEMM on the gathered rows of site ``site``, loading each token tile as soon
        as its rows have arrived."""
        from .. import ops

        x = self.sp_ag[site][:T]
        if mode == ops.EPI_SWIGLU_Q8:
            out = torch.empty(T, w.N // 2, dtype=x.dtype, device=x.device) if out is None else out
            f32, act = None, out
        else:
            out = torch.empty(T, w.N, dtype=torch.float32, device=x.device) if out is None else out
            f32, act = out, None
        require_ext().qgemm_sp(*w.args(), x, T, mode, f32, act, bias, out.stride(0), [], [], None, self.rank, 0, 0,
                               self.sp_ag_flags[site], self.sp_epoch[site:site + 1], self.wait_s)
        ops._count()
        return out

    def sp_reduce_norm_ag(self, site: int, x_loc: torch.Tensor, T: int, norm_w: torch.Tensor, eps: float,
                          reduce: bool = True, bias=None, self_only: bool = False) -> None:
        """Owner side of site ``site``: x_loc += the received partials (``reduce``), then RMSNorm rows
        pushed to every rank's gather buffer ``site`` (``self_only``: only into this rank's)."""
        from .. import ops

        C = require_ext()
        chunk = -(-T // self.world)
        H = x_loc.shape[1]
        C.sp_reduce_norm_ag(x_loc, T, self.rank, chunk, self.sp_slots if reduce else None,
                            self.sp_rs_flags[site] if reduce else None, self.world if reduce else 0,
                            self.sp_max_tiles, C.gemm_tile_rows(T), -(-H // 128), bias, norm_w, eps,
                            self._sp_ag[site], self._sp_agf[site], self.sp_epoch[site:site + 1],
                            self.sp_done[site:site + 1], self.wait_s, int(self.sp_act_dtype == torch.float16),
                            int(self_only))
        ops._count()

    def sp_gathered(self, site: int, T: int) -> torch.Tensor:
        """The gathered rows of site ``site`` once every rank's push has landed (device-side wait)."""
        from .. import ops

        require_ext().sp_ag_wait(self.sp_ag_flags[site], self.sp_epoch[site:site + 1], T, self.wait_s)
        ops._count()
        return self.sp_ag[site][:T]

    def push_ok(self, T: int, H: int) -> bool:
        return self.push_fused and T * H <= self.push_elems

    def push_args(self, j: int, T: int, H: int):
        """Arguments of ``ops.gemv_allreduce`` for call site j (0: attention output, 1: FFN down)."""
        if not self.push_ok(T, H):
            raise ValueError(f"fused GEMV all-reduce buffers hold {self.push_elems} values, {T * H} requested")
        return self._push_bufs[j], self.push_epoch, self.push_done, self.rank, self.wait_s, self.skip_signal

    def partial(self, j: int, T: int, H: int) -> torch.Tensor:
        """Local partial-sum buffer j (0: attention output, 1: FFN down) viewed as f32 [T, H]."""
        if T * H > self._n:
            raise ValueError(f"fused all-reduce buffer holds {self._n} values, {T * H} requested")
        return self.buf[j * self._n: j * self._n + T * H].view(T, H)

    def allreduce_add(self, j: int, x: torch.Tensor) -> None:
        """x += sum over ranks of partial buffer j (every rank calls it with its own x)."""
        n = x.numel()
        blocks = max(1, min(32, (n // 4 + 255) // 256))
        require_ext().allreduce_add(x, self._bufs[j], self._flags, self.epoch, self.rank, blocks, self.wait_s,
                                    int(self.skip_signal), self._mc_bufs[j])

    # ------------------------------------------------------------------ NCCL baseline
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(x, group=self.group)
        return x

    def all_gather_cols(self, y: torch.Tensor) -> torch.Tensor:
        """Concatenate every rank's [T, n_r] along columns (vocab-parallel logits; equal n_r)."""
        parts = [torch.empty_like(y) for _ in range(self.world)]
        dist.all_gather(parts, y.contiguous(), group=self.group)
        return torch.cat(parts, 1)

    def barrier(self) -> None:
        dist.barrier(group=self.group)

    def check(self) -> None:
        """Raise if a fused all-reduce gave up waiting for a peer (bounded device-side waits)."""
        from .. import ops

        err = ops.gemm_error()
        kind = err & 0xF00
        if kind == 0x300:
            raise RuntimeError(f"fused all-reduce: peer {err & 0xFF} did not arrive within the wait limit")
        if kind == 0x500:
            raise RuntimeError(f"fused reduce-scatter: rank {err & 0xFF}'s tiles did not arrive within the wait limit")
        if kind in (0x400, 0x600):
            raise RuntimeError("fused all-gather: a peer's rows did not arrive within the wait limit")
        if kind in (0x700, 0x800, 0x900):
            raise RuntimeError(f"expert all-to-all: rank {err & 0xFF} did not arrive within the wait limit")


def env_world() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), \
        int(os.environ.get("LOCAL_RANK", "0"))
