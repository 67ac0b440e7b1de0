"""Kernel microbenchmarks on Llama-3-8B shapes (random Q4_K / Q6_K weights), timed with CUDA events
around a CUDA graph of ``--iters`` launches (device time only, no host gaps).

    python -m barq_inference_b200.ops.kernel_bench gemm_gate_up --tokens 64
    python -m barq_inference_b200.ops.kernel_bench gemv_gate_up
    python -m barq_inference_b200.ops.kernel_bench all

Each case prints one line: name, microseconds per launch, GB/s of weight bytes, TFLOP/s.  The same
cases, run a few times without timing (``--iters 3 --no-graph``), are the profiling targets for ncu.
"""
from __future__ import annotations

import argparse
import os

import torch

from . import EPI_ADD_F32, EPI_STORE_F32, EPI_SWIGLU_Q8, QWeight, gemm, gemv, interleave_gate_up, quantize_q8


def _qw(N: int, K: int, t, seed: int = 0) -> QWeight:
    from ..gguf import quantize

    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.02
    return QWeight.from_packed(quantize(w, t), t, N, K, "cuda").finalize()


def _time(fn, iters: int, graph: bool) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    if graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        run = g.replay
    else:
        def run():
            for _ in range(iters):
                fn()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1e3


def cases(tokens: int):
    from ..gguf import GGMLType

    def gate_up():
        return interleave_gate_up(_qw(14336, 4096, GGMLType.Q4_K, 1), _qw(14336, 4096, GGMLType.Q4_K, 2)).finalize()

    def gemm_gate_up():
        w = gate_up()
        x = torch.randn(tokens, 4096, device="cuda").half()
        return w, (lambda: gemm(w, x, EPI_SWIGLU_Q8)), 2.0 * tokens * w.N * w.K

    def gemm_down():
        w = _qw(4096, 14336, GGMLType.Q4_K, 3)
        x = torch.randn(tokens, 14336, device="cuda").half()
        out = torch.zeros(tokens, 4096, device="cuda")
        return w, (lambda: gemm(w, x, EPI_ADD_F32, out=out)), 2.0 * tokens * w.N * w.K

    def gemv_gate_up():
        w = gate_up()
        xa = quantize_q8(torch.randn(1, 4096, device="cuda"), True)
        return w, (lambda: gemv(w, xa, 1, EPI_SWIGLU_Q8, x2=True)), 2.0 * w.N * w.K

    def gemv_head():
        w = _qw(128256, 4096, GGMLType.Q6_K, 4)
        xa = quantize_q8(torch.randn(1, 4096, device="cuda"), True)
        out = torch.empty(1, w.N, device="cuda")
        return w, (lambda: gemv(w, xa, 1, EPI_STORE_F32, out=out, x2=True)), 2.0 * w.N * w.K

    def gemv_qkv():
        w = _qw(6144, 4096, GGMLType.Q4_K, 5)
        xa = quantize_q8(torch.randn(1, 4096, device="cuda"), True)
        out = torch.empty(1, w.N, device="cuda")
        return w, (lambda: gemv(w, xa, 1, EPI_STORE_F32, out=out, x2=True)), 2.0 * w.N * w.K

    def gemv_o_tp2(push: bool):
        # attention output of one rank under TP=2 (K halved); push: the all-reduce fused in, as a
        # world of one (the exchange protocol runs against this GPU's own flag)
        def make():
            from . import gemv_allreduce

            w = _qw(4096, 2048, GGMLType.Q4_K, 6)
            xa = quantize_q8(torch.randn(1, 2048, device="cuda"), True)
            x = torch.zeros(1, 4096, device="cuda")
            if not push:
                return w, (lambda: gemv(w, xa, 1, EPI_ADD_F32, out=x, x2=True)), 2.0 * w.N * w.K
            buf = torch.zeros(4096, dtype=torch.int64, device="cuda")
            ctr = torch.zeros(2, dtype=torch.int32, device="cuda"), torch.zeros(2, dtype=torch.int32, device="cuda")
            tab = torch.tensor([buf.data_ptr()], dtype=torch.int64, device="cuda")
            args = lambda j, T, H: (tab, ctr[0], ctr[1], 0, 5.0, 0)  # noqa: E731
            return w, (lambda: gemv_allreduce(w, xa, 1, x, args, 0)), 2.0 * w.N * w.K
        return make

    def allreduce_w1():
        # the separate one-shot all-reduce kernel on a decode-sized message, as a world of one
        from . import require_ext

        x = torch.zeros(1, 4096, device="cuda")
        buf = torch.zeros(4096, device="cuda")
        flags = torch.zeros(64 * 8, dtype=torch.int32, device="cuda")
        epoch = torch.zeros(64, dtype=torch.int32, device="cuda")
        C = require_ext()
        fn = lambda: C.allreduce_add(x, [buf.data_ptr()], [flags.data_ptr()], epoch, 0, 4, 5.0, 0, 0)  # noqa: E731
        return _qw(128, 256, GGMLType.Q4_K, 7), fn, 0.0

    def decode_step(B: int, ctx: int):
        # one whole decode step of Llama-3-8B (random Q4_K / Q6_K weights) over B sequences of
        # ctx cached tokens each, eager launches: the launch-list target for "where does a decode
        # step's time go"
        def make():
            from ..models import POLICIES, preset, random_tensors
            from ..models.runner import LlamaRunner, StepInput

            cfg = preset("llama3-8b")
            r = LlamaRunner(cfg, random_tensors(cfg, POLICIES["llama3-8b"], seed=0, device="cuda"), "cuda")
            pages = ctx // 16 + 2
            r.allocate_kv(1 + B * pages)
            tables = torch.arange(1, 1 + B * pages, dtype=torch.int32, device="cuda").view(B, pages)

            def inp(seqs, start, T):
                pos = torch.arange(start, start + T, dtype=torch.int32, device="cuda").repeat(len(seqs))
                sq = torch.tensor(seqs, device="cuda").repeat_interleave(T)
                bt = tables[sq.unique_consecutive()]
                row = torch.arange(len(seqs), device="cuda").repeat_interleave(T)
                slots = bt[row, pos.long() // 16].long() * 16 + pos.long() % 16
                ids = torch.randint(0, cfg.vocab, (len(seqs) * T,), device="cuda", dtype=torch.int32)
                return StepInput(ids, pos, slots, bt.contiguous(),
                                 torch.full((len(seqs),), start + T, dtype=torch.int32, device="cuda"),
                                 (torch.arange(len(seqs), device="cuda") + 1) * T - 1, T == 1,
                                 q_start=torch.arange(len(seqs) + 1, dtype=torch.int32, device="cuda") * T, max_q=T)

            for b0 in range(0, B, 8):  # prefill the contexts 8 sequences at a time
                r.forward(inp(list(range(b0, min(B, b0 + 8))), 0, ctx))
            step = inp(list(range(B)), ctx, 1)  # rewrites the same positions each call
            return _qw(128, 256, GGMLType.Q4_K, 8), (lambda: r.forward(step)), 0.0
        return make

    def attn_decode(B: int, ctx: int):
        # one layer's decode attention of Llama-3-8B shapes: B sequences of ctx tokens, 32 query /
        # 8 KV heads of 128, fp16 paged KV (16-token pages, scattered); bytes = the K/V stream
        def make():
            from . import decode_attention

            H, Hkv, D = 32, 8, 128
            pages = (ctx + 15) // 16
            nb = B * pages + 1
            kc = torch.randn(nb, Hkv, 16, D, device="cuda").half()
            vc = torch.randn(nb, Hkv, 16, D, device="cuda").half()
            bt = (torch.randperm(nb - 1, device="cuda")[: B * pages] + 1).int().view(B, pages)
            lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
            q = torch.randn(B, H, D, device="cuda").bfloat16()

            class _W:  # bytes streamed per call, for the GB/s column
                @staticmethod
                def nbytes():
                    return B * ctx * Hkv * D * 2 * 2
            sp = int(os.environ.get("BARQ_BENCH_SPLITS", "0")) or None  # sweep knob of this case
            return _W, (lambda: decode_attention(q, kc, vc, bt, lens, H, Hkv, D, D ** -0.5, splits=sp)), \
                4.0 * B * H * ctx * D
        return make

    class _Bytes:  # bytes an op must move, for the GB/s column of cases without a weight
        def __init__(self, n):
            self.n = n

        def nbytes(self):
            return self.n

    def rope_kv(T: int):
        # RoPE + K/V cache write of one Llama-3-8B layer for T tokens (qkv f32 in, q bf16 + K/V fp16 out)
        def make():
            from . import rope_kv_write
            from ..models import preset
            from ..models.rope import rope_cos_sin

            cfg = preset("llama3-8b")
            H, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
            qkv = torch.randn(T, (H + 2 * Hkv) * D, device="cuda")
            cos, sin = rope_cos_sin(cfg, 4096, "cuda")
            pos = torch.arange(T, dtype=torch.int32, device="cuda") + 1000
            slots = torch.arange(T, device="cuda") * 16 + 16  # one page per token row
            kc = torch.zeros(T + 2, Hkv, 16, D, device="cuda").half()
            vc = torch.zeros_like(kc)
            nb = qkv.numel() * 4 + T * H * D * 2 + 2 * T * Hkv * D * 2
            return _Bytes(nb), (lambda: rope_kv_write(qkv, pos, slots, cos, sin, H, Hkv, D, cfg.rot_dim,
                                                      cfg.rope_neox, kc, vc)), 0.0
        return make

    def sampler(B: int):
        # fused sampler over a 128256-token vocabulary: top-k 40, top-p 0.95, temperature 0.8
        def make():
            from . import sample

            V = 128256
            lg = torch.randn(B, V, device="cuda")
            f = lambda v, dt=torch.float32: torch.full((B,), v, dtype=dt, device="cuda")  # noqa: E731
            args = (f(0.8), f(40, torch.int32), f(0.95), f(0.0), f(7, torch.int64), f(0, torch.int32))
            return _Bytes(lg.numel() * 4), (lambda: sample(lg, *args)), 0.0
        return make

    def prefill_attn(T: int):
        # causal prefill attention of one Llama-3-8B layer over a T-token prompt (fp16 paged KV)
        def make():
            from . import prefill_attention

            H, Hkv, D = 32, 8, 128
            pages = (T + 15) // 16
            kc = torch.randn(pages + 1, Hkv, 16, D, device="cuda").half()
            vc = torch.randn_like(kc)
            bt = torch.arange(1, pages + 1, dtype=torch.int32, device="cuda").view(1, pages)
            q = torch.randn(T, H, D, device="cuda").bfloat16()
            qs = torch.tensor([0, T], dtype=torch.int32, device="cuda")
            cl = torch.tensor([T], dtype=torch.int32, device="cuda")
            flops = 4.0 * H * D * T * T / 2
            return _Bytes(2 * T * Hkv * D * 2 + 2 * T * H * D * 2), (lambda: prefill_attention(
                q, kc, vc, bt, qs, cl, T, H, Hkv, D, D ** -0.5)), flops
        return make

    def moe_layer(T: int):
        # one Mixtral-shaped MoE FFN (8 experts of 4096 -> 14336, top-2, Q4_K) for T tokens on one GPU:
        # router matmul, routing kernels, grouped gate|up and down tcgen05 GEMMs, combine
        def make():
            import dataclasses

            from ..models import POLICIES, preset, random_tensors
            from ..models.moe import MoEBlock

            cfg = dataclasses.replace(preset("mixtral-8x7b"), n_layers=1)
            tensors = random_tensors(cfg, POLICIES["mixtral-8x7b"], seed=0, device="cuda")
            blk = MoEBlock(cfg, tensors, "blk.0.", "cuda")
            del tensors
            hb = torch.randn(T, cfg.hidden, device="cuda").half()
            x = torch.zeros(T, cfg.hidden, device="cuda")

            class _R:
                ser_threshold, fused_moe, x2 = 0.0, True, True
            nb = blk.gate_up.nbytes() + blk.down.nbytes()
            return _Bytes(nb), (lambda: blk.forward(_R(), None, hb, T, x)), 2.0 * T * 2 * 3 * 4096 * 14336
        return make

    def mla_decode(B: int, ctx: int):
        # DeepSeek-V2-Lite MLA decode attention: B rows of ctx cached latents (576-wide bf16 rows), 16 heads
        def make():
            from . import mla_attention

            H, qdim = 16, 192
            pages = (ctx + 15) // 16
            cache = torch.randn(B * pages + 1, 16, 576, device="cuda").bfloat16()
            bt = (torch.arange(B * pages, dtype=torch.int32, device="cuda") + 1).view(B, pages)
            q_lat = torch.randn(B, H, 512, device="cuda")
            q = torch.randn(B, H * qdim, device="cuda")
            rs = torch.arange(B, dtype=torch.int32, device="cuda")
            rl = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
            splits = max(1, min(32, -(-2 * 148 // B)))
            return _Bytes(B * ctx * 576 * 2), (lambda: mla_attention(q_lat, q, qdim, 128, cache, bt, rs, rl, H, splits,
                                                                      0.1)), 4.0 * B * H * ctx * 576
        return make

    def sp_reduce(T: int):
        # owner side of a sequence-parallel site as a world of one rank (Llama-3-8B hidden 4096): wait
        # for the pushed tiles, add them into the residual rows, RMSNorm, push the rows and their flags
        def make():
            from . import require_ext

            C = require_ext()
            H = 4096
            max_tiles = (H // 128) * ((T + 31) // 32)
            slots = torch.randn(T * H, device="cuda")
            flags = torch.full((max_tiles,), 1 << 30, dtype=torch.int32, device="cuda")  # every tile "arrived"
            x = torch.randn(T, H, device="cuda")
            nw = torch.ones(H, device="cuda")
            ag = torch.empty(T, H, dtype=torch.float16, device="cuda")
            agf = torch.zeros(T, dtype=torch.int32, device="cuda")
            ep = torch.zeros(1, dtype=torch.int32, device="cuda")
            done = torch.zeros(1, dtype=torch.int32, device="cuda")

            def run():
                C.sp_reduce_norm_ag(x, T, 0, T, slots, flags, 1, max_tiles, C.gemm_tile_rows(T), H // 128, None, nw,
                                    1e-5, [ag.data_ptr()], [agf.data_ptr()], ep, done, 5.0, 1, 0)
            return _Bytes(T * H * (4 + 4 + 4 + 2)), run, 0.0
        return make

    return {"allreduce_w1": allreduce_w1, "attn_decode_bs32": attn_decode(32, 1024),
            "mla_decode_bs32": mla_decode(32, 4096), "sp_reduce_t512": sp_reduce(512),
            "rope_kv_t32": rope_kv(32), "sampler_bs32": sampler(32), "prefill_attn_t2048": prefill_attn(2048),
            "moe_mixtral_t64": moe_layer(64),
            "attn_decode_bs1": attn_decode(1, 1024), "decode_step_bs1": decode_step(1, 64),
            "decode_step_bs32": decode_step(32, 1024), "decode_step_bs64": decode_step(64, 1024), "gemm_gate_up": gemm_gate_up, "gemm_down": gemm_down, "gemv_gate_up": gemv_gate_up,
            "gemv_head": gemv_head, "gemv_qkv": gemv_qkv, "gemv_o_tp2": gemv_o_tp2(False),
            "gemv_o_tp2_push": gemv_o_tp2(True)}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("case", help="case name or 'all'")
    ap.add_argument("--tokens", type=int, default=64, help="token rows for the GEMM cases")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-graph", action="store_true", help="plain launches (for profilers)")
    a = ap.parse_args(argv)
    cs = cases(a.tokens)
    names = list(cs) if a.case == "all" else [a.case]
    for n in names:
        w, fn, flops = cs[n]()
        us = _time(fn, a.iters, not a.no_graph)
        gbs = w.nbytes() / us / 1e3
        print(f"{n}: {us:.1f} us  {gbs:.0f} GB/s  {flops / us / 1e6:.1f} TFLOP/s", flush=True)
        del w, fn
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
