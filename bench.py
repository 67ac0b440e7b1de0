"""Headline benchmark on the Llama-3-8B architecture (Q4_K, Q6_K head), random-init weights and
uniform-random prompt ids (no checkpoint or dataset is available offline):

  (b) the value: decode tok/s of 32 concurrent requests with 1024-token prompts, 256 decode tokens
      each, paged KV in 16-token fp16 blocks (W warm-up steps, then K timed steps);
  (a) extra: batch 1 with a 512-token prompt and 256 greedy decode tokens (decode tok/s), and the
      p50 time to first token of that prompt;
  plus the prefill tok/s of the 32 x 1024 prompts.

    python bench.py --gpus N --steps K --warmup W           (N > 1: one process per GPU via torchrun)
    python bench.py --impl reference ...                     (reference arm)

Multi-GPU (default ``--parallel tp``): ONE engine tensor-parallel over all N GPUs (strong scaling:
the same requests, the row-parallel all-reduces fused into the GEMV / GEMM kernels over NVLink);
``--parallel dp`` runs an independent replica per GPU instead (weak scaling).  Times are taken on
the device with CUDA events, max over ranks.  A "step" is one continuous-batching decode step of
the engine's public ``step()`` API: it includes the host->device copy of the step's inputs from
pinned memory, the CUDA-graph replay (embedding .. sampling) and the device->host read of the
sampled ids.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (bs1, bs64) + prefill tok/s + p50 TTFT at 1/2/4/8 B200, max over ranks"
MODELS = {"llama3-8b": "Llama-3-8B (Q4_K, Q6_K output), random-init",
          "llama3-70b": "Llama-3-70B (Q4_K, Q6_K attention and output, YaRN x4), random-init",
          "mixtral-8x7b": "Mixtral-8x7B (Q4_K, Q6_K output), random-init",
          "deepseek-v2-lite": "DeepSeek-V2-Lite (Q4_K experts, Q8_0 attention), random-init"}
DECODE_TOKENS = 256  # decode tokens per request in every BASELINE workload


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=240)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="barq", choices=["barq", "reference"])
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--ttft-prompt", type=int, default=512)
    ap.add_argument("--ttft-reps", type=int, default=5)
    ap.add_argument("--bs1-steps", type=int, default=DECODE_TOKENS)
    ap.add_argument("--e2e-tokens", type=int, default=32)
    ap.add_argument("--layers", type=int, default=0, help="override layer count (debug only; invalid for the headline)")
    ap.add_argument("--batch-per-gpu", action="store_true",
                    help="with --parallel tp: --batch requests per GPU (global batch = batch x N, weak scaling); "
                         "default: --batch is the global batch (strong scaling)")
    ap.add_argument("--parallel", default="tp", choices=["dp", "tp"],
                    help="tp: one tensor-parallel engine over all GPUs (strong scaling, default); dp: one engine "
                         "replica per GPU (weak scaling)")
    ap.add_argument("--ser", type=float, default=0.0,
                    help="MoE smart expert reduction: drop a routed expert whose gate weight is below this")
    ap.add_argument("--no-fmoe", action="store_true", help="MoE: per-expert loop instead of the fused path")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                    help="tp all-reduce: fused one-shot kernel over NVLink peer memory, or NCCL")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def reference_arm(args):
    why = ("the reference (YASSERRMD/barq-inference) is a pure-Rust Cargo workspace with no Python package "
           "and no Rust toolchain on this image (pip install: 'Neither setup.py nor pyproject.toml found'); "
           "its CUDA backend launches no kernels (host fallbacks) and has no multi-GPU path")
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        return reference_arm(args)
    import numpy as np
    import torch
    import torch.distributed as dist

    from barq_inference_b200 import ops
    from barq_inference_b200.engine.engine import Engine, EngineConfig
    from barq_inference_b200.engine.sampling_params import SamplingParams
    from barq_inference_b200.models import POLICIES, preset, random_tensors

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)

    cfg = preset(args.model)
    if args.layers:
        cfg.n_layers = args.layers
    t_init = time.time()
    tensors = random_tensors(cfg, POLICIES[args.model], seed=0, device=dev)
    tp = world if args.parallel == "tp" else 1
    weak_tp = tp > 1 and args.batch_per_gpu
    B, P = args.batch * (world if weak_tp else 1), args.prompt_len
    max_len = P + args.warmup + args.steps + args.e2e_tokens + 64
    max_len = max(max_len, args.ttft_prompt + args.bs1_steps + 16)
    max_len = (max_len + 15) // 16 * 16
    blocks_needed = B * (max_len // 16 + 2) + 64
    ec = EngineConfig(max_num_seqs=max(B, 1), max_num_batched_tokens=8192, max_model_len=max_len,
                      num_blocks=blocks_needed, cuda_graphs=True, tp=tp, fused_comm=args.comm == "fused",
                      ser_threshold=args.ser, fused_moe=not args.no_fmoe)
    eng = Engine(cfg, tensors, ec)
    del tensors
    torch.cuda.empty_cache()
    init_s = time.time() - t_init
    rng = np.random.default_rng(1 + (rank if tp == 1 else 0))  # TP ranks serve the same requests
    mult = world if tp == 1 else 1  # DP: aggregate over replicas; TP: one engine
    greedy = lambda n: SamplingParams.greedy_params(max_tokens=n, ignore_eos=True)  # noqa: E731

    def ev():
        return torch.cuda.Event(enable_timing=True)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- (1) TTFT of a 512-token prompt at batch 1, then batch-1 decode
    ttfts = []
    for r in range(args.ttft_reps + 1):
        seq = eng.add_request(rng.integers(0, cfg.vocab, args.ttft_prompt).tolist(), greedy(args.bs1_steps + 2))
        barrier()
        e0, e1 = ev(), ev()
        e0.record()
        while not seq.output:
            eng.step()
        e1.record()
        torch.cuda.synchronize()
        if r > 0:
            ttfts.append(e0.elapsed_time(e1))
        if r < args.ttft_reps:
            while not seq.finished:
                eng.step()
    # seq (last) continues: batch-1 decode
    for _ in range(4):
        eng.step()
    barrier()
    e0, e1 = ev(), ev()
    e0.record()
    n1 = 0
    while not seq.finished and n1 < args.bs1_steps - 6:
        eng.step()
        n1 += 1
    e1.record()
    torch.cuda.synchronize()
    bs1_ms = max_over_ranks(e0.elapsed_time(e1) / max(1, n1))
    bs1_replay_ms = None
    if 1 in eng.graphs:  # device time of the batch-1 step alone (back-to-back graph replays)
        g1 = eng.graphs[1].graph
        g1.replay()
        barrier()
        r0, r1 = ev(), ev()
        r0.record()
        for _ in range(10):
            g1.replay()
        r1.record()
        torch.cuda.synchronize()
        bs1_replay_ms = max_over_ranks(r0.elapsed_time(r1) / 10)
    while eng.has_work():
        eng.step()

    # ---- (2) batch-B prefill of P-token prompts
    seqs = [eng.add_request(rng.integers(0, cfg.vocab, P).tolist(), greedy(max(DECODE_TOKENS, args.warmup + args.steps + 4)))
            for _ in range(B)]
    barrier()
    e0, e1 = ev(), ev()
    e0.record()
    while any(not s.output for s in seqs):
        eng.step()
    e1.record()
    torch.cuda.synchronize()
    prefill_ms = max_over_ranks(e0.elapsed_time(e1))

    # ---- (3) timed decode steps at batch B
    for _ in range(args.warmup):
        eng.step()
    launches0 = ops.LAUNCHES[0]
    clocks = ClockSampler(local)
    barrier()
    clocks.start()
    e0, e1 = ev(), ev()
    e0.record()
    for _ in range(args.steps):
        eng.step()
    e1.record()
    barrier()
    ck = clocks.stop()
    dec_ms = max_over_ranks(e0.elapsed_time(e1))
    # device time of the decode step alone: back-to-back replays of the captured graph (no host work
    # in between); ms_per_step minus this is the engine's host overhead per step
    replay_ms = None
    if eng.graphs:
        gb = eng.graphs[max(eng.graphs)]
        gb.graph.replay()
        barrier()
        r0, r1 = ev(), ev()
        r0.record()
        for _ in range(10):
            gb.graph.replay()
        r1.record()
        torch.cuda.synchronize()
        replay_ms = max_over_ranks(r0.elapsed_time(r1) / 10)
    while eng.has_work():
        eng.step()
    # kernel launches per decode step: one eager (non-graph) forward of the same batch, counted
    eng.ecfg.cuda_graphs = False
    probe = [eng.add_request(rng.integers(0, cfg.vocab, 16).tolist(), greedy(3)) for _ in range(B)]
    while any(not s.output for s in probe):
        eng.step()
    c0 = ops.LAUNCHES[0]
    eng.step()
    launches_per_step = ops.LAUNCHES[0] - c0
    while eng.has_work():
        eng.step()
    eng.ecfg.cuda_graphs = True

    # ---- (4) end to end through the public generate() API (host clock, includes H2D + D2H every step)
    prompts = [rng.integers(0, cfg.vocab, P).tolist() for _ in range(B)]
    eng.timings = {k: 0 for k in eng.timings}
    barrier()
    t0 = time.perf_counter()
    res = eng.generate(prompts, greedy(args.e2e_tokens))
    torch.cuda.synchronize()
    t_e2e = time.perf_counter() - t0
    e2e_dec = eng.timings["decode_tokens"] / max(1e-9, eng.timings["decode_s"])
    e2e_dec = max_over_ranks(-e2e_dec) * -1 if world > 1 else e2e_dec  # slowest rank
    # per decode step: ONE host->device copy of the packed inputs of the graph bucket, one read of
    # the sampled ids
    gbB = eng.graphs.get(next((b for b in eng.ecfg.graph_buckets if b >= B), B))
    h2d = gbB.packed.nbytes if gbB is not None else B * (40 + 4 * eng.max_blocks_per_seq)
    d2h = B * 4

    if rank == 0:
        value = mult * B * args.steps / (dec_ms / 1e3)
        out = {
            "metric": METRIC,
            "value": round(value, 2),
            "unit": ("tokens/s (decode, batch %d per GPU, aggregate)" % B) if tp == 1 else
                    ("tokens/s (decode, batch %d%s, tensor parallel over %d GPUs)"
                     % (B, " = %d per GPU" % args.batch if weak_tp else "", world)),
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dec_ms / args.steps, 4),
            "higher_is_better": True,
            "scaling": "weak" if tp == 1 or weak_tp else "strong",
            "vs_baseline": None,
            "dtype": "Q4_K/Q6_K weights dequantized in-kernel; decode GEMV activations two-term int8 (~15-bit: "
                     "x = d*q + dl*ql), prefill / batched GEMM activations bf16 on tcgen05; fp32 accumulation and "
                     "residual stream; fp16 KV",
            "data": "synthetic: random-init N(0,0.02) weights quantized to Q4_K/Q6_K, uniform-random prompt ids",
            "config": {"model": MODELS.get(args.model, args.model) + (f" ({cfg.n_layers} layers)" if args.layers else ""), "global_batch": B * mult,
                       "seq_len": P, "parallelism": (f"dp{world}" if tp == 1 else f"tp{world}-{args.comm}") +
                       (f"-ser{args.ser}" if args.ser else "") + ("-nofmoe" if args.no_fmoe else ""),
                       "l2": "inputs larger than L2 (4.6 GB of weights streamed per step)"},
            "extra": {
                "decode_tok_s_bs1": round(mult * 1e3 / bs1_ms, 2),
                "prefill_tok_s": round(mult * B * P / (prefill_ms / 1e3), 1),
                "ttft_p50_ms_512": round(statistics.median(ttfts), 3) if ttfts else None,
                "init_s": round(init_s, 1),
                "decode_graph_replay_ms": round(replay_ms, 4) if replay_ms is not None else None,
                "bs1_graph_replay_ms": round(bs1_replay_ms, 4) if bs1_replay_ms is not None else None,
            },
            "e2e": {"value": round(mult * e2e_dec, 2), "unit": "tokens/s decode via Engine.generate()",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "wall_s": round(t_e2e, 3), "tokens": sum(len(r.tokens) for r in res)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": ck,
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        if tp > 1:
            # captured CUDA graphs hold NCCL collectives: tearing the communicator down under them can
            # block; every result is printed, so synchronize the ranks and leave without teardown
            dist.barrier()
            torch.cuda.synchronize()
            sys.stdout.flush()
            os._exit(0)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
