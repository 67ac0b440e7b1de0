"""The inference engine: model runner + paged KV + scheduler + device sampler + CUDA graphs.

Public API (what the CLI, the HTTP/UDS servers and ``bench.py`` call):

* ``Engine.from_gguf(path, ...)`` / ``Engine(cfg, tensors, ...)``
* ``Engine.generate(prompts, params) -> list[GenerationResult]`` (batched, blocking)
* ``Engine.add_request(prompt, params, on_token=...)`` + ``Engine.step()`` (streaming / serving)

Parity: ``ModelContext::{encode, decode, sample, generate}`` (``models/src/context.rs:391-556``),
``BatchEngine::run`` (``advanced/src/batch_engine.rs:106-191``, whose forward samples random
logits) and the CUDA-graph flag (``cli/src/performance.rs:16-22``, env var only).  Here decode steps
are captured once per batch-size bucket as CUDA graphs (embedding through sampling), prompts are
prefilled in chunks, and tokens stream out one step at a time.
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import ops
from ..models.config import ModelConfig
from ..models.runner import LlamaRunner, StepInput
from .kv_cache import BlockManager, new_block_manager  # noqa: F401
from .logprobs import record_logprobs
from .scheduler import ScheduledStep, SchedulerConfig, new_scheduler
from .sampling_params import SamplingParams
from .sequence import Sequence


@dataclass
class EngineConfig:
    max_num_seqs: int = 64
    max_num_batched_tokens: int = 8192
    max_model_len: int = 4096
    block_size: int = 16
    num_blocks: int | None = None   # None -> sized from kv_cache_gb
    kv_cache_gb: float = 8.0
    kv_dtype: str = "fp16"          # fp16 | bf16 | fp8 (e4m3 with one f32 scale per stored row)
    cuda_graphs: bool = True
    graph_buckets: tuple[int, ...] = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)
    prefix_caching: bool = False
    chunked_prefill: bool = True
    device: str = "cuda"
    ser_threshold: float = 0.0      # MoE smart expert reduction (--ser)
    fused_moe: bool = True          # --fmoe
    act_x2: bool = True             # two-term int8 decode activations (False: single int8 term)
    tp: int = 1                     # tensor parallel degree (one process per GPU, torch.distributed)
    pp: int = 1                     # pipeline stages (one process per GPU, contiguous layer ranges)
    rank_timeout_s: float = 30.0    # TP: a peer without a heartbeat for this long fails the step
    fused_comm: bool = True         # TP: fused one-shot all-reduce kernel (False: NCCL all-reduce)
    max_waiting: int = 0            # admission control: refuse requests beyond this queue depth (0: off)

    @staticmethod
    def preset(name: str, **kw) -> "EngineConfig":
        """CLI presets (``cli/src/main.rs`` --preset) mapped to concrete switches."""
        base = {
            "max-speed": dict(cuda_graphs=True, kv_dtype="fp16", max_num_seqs=128),
            "balanced": dict(cuda_graphs=True, kv_dtype="fp16"),
            "max-quality": dict(cuda_graphs=True, kv_dtype="bf16"),
            "gpu": dict(cuda_graphs=True),
            "cpu": dict(cuda_graphs=False),
        }[name]
        base.update(kw)
        return EngineConfig(**base)


@dataclass
class GenerationResult:
    prompt: list[int]
    tokens: list[int]
    finish_reason: str
    ttft_s: float | None
    latency_s: float
    logprobs: list[float] = field(default_factory=list)
    top_logprobs: list[list[tuple[int, float]]] = field(default_factory=list)


class _GraphBucket:
    __slots__ = ("B", "graph", "out_ids", "packed")


class Engine:
    def __init__(self, cfg: ModelConfig, tensors, engine_cfg: EngineConfig | None = None, runner=None):
        self.cfg = cfg
        self.ecfg = ec = engine_cfg or EngineConfig()
        self.device = torch.device(ec.device)
        kv_dtype = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp8": torch.float8_e4m3fn}[ec.kv_dtype]
        self.runner = runner or make_runner(cfg, tensors, self.device, kv_dtype, ec)
        self.max_blocks_per_seq = (ec.max_model_len + ec.block_size - 1) // ec.block_size
        nb = ec.num_blocks
        if nb is None:
            nb = max(64, int(ec.kv_cache_gb * (1 << 30) // self.runner.kv_bytes_per_block(ec.block_size)))
        self.runner.allocate_kv(nb, ec.block_size)
        from ..utils.trace import StepProfiler

        self._profile = StepProfiler.from_env(self)  # BARQ_PROFILE / BARQ_NVTX
        self.last_plan = None
        self.blocks = new_block_manager(nb, ec.block_size)  # C++ pool when built
        self.dummy_block = self.blocks.allocate(1)[0]  # padding rows of graph batches write here
        self.prefix_cache = None
        if ec.prefix_caching:
            from .prefix_cache import new_prefix_cache

            self.prefix_cache = new_prefix_cache(self.blocks)
        self.sched = new_scheduler(SchedulerConfig(ec.max_num_seqs, ec.max_num_batched_tokens, ec.max_model_len,
                                               ec.chunked_prefill, sliding_window=cfg.sliding_window,
                                               max_waiting=ec.max_waiting),
                               self.blocks, self.prefix_cache)
        self.sched.dummy_block = self.dummy_block
        self.graphs: dict[int, _GraphBucket] = {}
        self.metrics = None
        self.step_count = 0
        self.timings = {"prefill_s": 0.0, "decode_s": 0.0, "prefill_tokens": 0, "decode_tokens": 0}

    # ------------------------------------------------------------------ construction helpers
    @staticmethod
    def from_gguf(path: str, engine_cfg: EngineConfig | None = None, device: str | None = None) -> "Engine":
        from ..gguf import read_gguf_split as read_gguf
        from ..models.config import attach_rope_factors, config_from_gguf
        from ..models.weights import tensors_from_gguf

        g = read_gguf(path)
        cfg = attach_rope_factors(config_from_gguf(g.metadata, set(g.tensors)), g)
        ec = engine_cfg or EngineConfig()
        if device:
            ec.device = device
        ec.max_model_len = min(ec.max_model_len, cfg.max_ctx)
        tensors = tensors_from_gguf(g, device="cpu")
        eng = Engine(cfg, tensors, ec)
        eng.gguf = g
        return eng

    # ------------------------------------------------------------------ request API
    def add_request(self, prompt: list[int], params: SamplingParams | None = None, request_id: str = "",
                    on_token=None, embeds: tuple[int, torch.Tensor] | None = None) -> Sequence:
        """``embeds``: (first position, [n, hidden] tensor) input embeddings that replace the token
        embeddings of prompt positions first..first+n-1 (image patches of a multimodal prompt)."""
        params = params or SamplingParams()
        seq = Sequence(list(prompt), params, request_id=request_id, on_token=on_token)
        if embeds is not None:
            st, e = embeds
            if e.dim() != 2 or e.shape[1] != self.cfg.hidden or st < 0 or st + e.shape[0] > len(prompt):
                raise ValueError("embeds: need [n, hidden] rows inside the prompt")
            seq.embeds = (int(st), e.to(self.device, torch.float32))
        inj = getattr(self.runner, "injector", None)
        if inj is not None and inj.active("corrupt", self.step_count):  # fault injection: a bad request
            seq.prompt.append(self.cfg.vocab)
        if any(t < 0 or t >= self.cfg.vocab for t in seq.prompt):
            raise ValueError("prompt token id out of range")
        if params.grammar or params.json_mode or params.json_schema:
            from ..sampling.grammar_engine import make_grammar_state

            seq.grammar_state = make_grammar_state(self, params)
        if params.needs_host_sampler:
            from ..sampling.host_samplers import new_host_sampler

            seq.host_sampler = new_host_sampler(params, self.cfg.vocab)
        self.sched.add(seq)
        return seq

    def has_work(self) -> bool:
        return self.sched.has_work

    def abort(self, seq: Sequence) -> bool:
        """Stop generating for ``seq`` (e.g. its client disconnected); no further tokens are sent."""
        seq.on_token = None
        return self.sched.abort(seq)

    def embed(self, prompts: list[list[int]], normalize: bool = True) -> torch.Tensor:
        """Mean-pooled final-norm hidden states of each prompt ([N, hidden], fp32, on the CPU)."""
        from .embeddings import embed_gpu

        return embed_gpu(self, prompts, normalize)

    def generate(self, prompts: list[list[int]], params: SamplingParams | list[SamplingParams] | None = None
                 ) -> list[GenerationResult]:
        if params is None or isinstance(params, SamplingParams):
            params = [params or SamplingParams()] * len(prompts)
        seqs = [self.add_request(p, sp) for p, sp in zip(prompts, params)]
        while self.sched.has_work:
            self.step()
        return [self._result(s) for s in seqs]

    def _result(self, s: Sequence) -> GenerationResult:
        return GenerationResult(s.prompt, s.output, s.finish_reason or "", s.ttft,
                                (s.finish_time or time.perf_counter()) - s.arrival, s.logprobs, s.top_logprobs)

    # ------------------------------------------------------------------ one engine step
    def step(self) -> list[Sequence]:
        if self._profile is not None:
            return self._profile.step(self._step)
        return self._step()

    def _step(self) -> list[Sequence]:
        health = getattr(self.runner, "health", None)
        if health is not None:  # tensor parallel: every peer must be alive before a collective
            inj = self.runner.injector
            inj.on_step(self.step_count)
            health.check()
            if self.runner.comm is not None:
                self.runner.comm.skip_signal = inj.active("skip_flag", self.step_count)
        plan = self.sched.schedule()
        self.last_plan = plan
        if plan is None:
            if self.sched.waiting:
                raise RuntimeError("KV cache too small for the waiting request")
            return []
        t0 = time.perf_counter()
        if plan.kind == "decode":
            ids = self._run_decode(plan)
        else:
            ids = self._run_prefill(plan)
        dt = time.perf_counter() - t0
        key = "decode" if plan.kind == "decode" else "prefill"
        self.timings[key + "_s"] += dt
        self.timings[key + "_tokens"] += sum(plan.n_new)
        self.step_count += 1
        comm = getattr(self.runner, "comm", None)
        if comm is not None and comm.fused:
            comm.check()  # a peer that stopped answering raises here instead of slowing every step
        return self._commit(plan, ids)

    def _commit(self, plan: ScheduledStep, ids: list[int | None]) -> list[Sequence]:
        now = time.perf_counter()
        done = []
        for s, n, tok in zip(plan.seqs, plan.n_new, ids):
            s.n_cached += n
            if tok is None:  # prefill chunk that did not reach the end of the prompt
                continue
            if s.first_token_time is None:
                s.first_token_time = now
            s.output.append(tok)
            if s.grammar_state is not None:
                s.grammar_state.accept(tok)
            if s.on_token is not None:
                s.on_token(s, tok)
            reason = self._stop_reason(s, tok)
            if reason:
                s.finish_time = now
                self.sched.finish(s, reason)
                done.append(s)
                if s.on_token is not None:
                    s.on_token(s, -1)
        return done

    def _stop_reason(self, s: Sequence, tok: int) -> str | None:
        p = s.params
        if not p.ignore_eos and tok in self.cfg.eos_ids:
            return "stop"
        if tok in p.stop_token_ids:
            return "stop"
        if s.grammar_state is not None and s.grammar_state.done():
            return "stop"
        if len(s.output) >= p.max_tokens:
            return "length"
        if s.n_tokens >= self.ecfg.max_model_len:
            return "length"
        return None

    # ------------------------------------------------------------------ input building
    def _pinned(self, arr: np.ndarray) -> torch.Tensor:
        return torch.from_numpy(arr).pin_memory() if self.device.type == "cuda" else torch.from_numpy(arr)

    def _stage(self, key: str, arr: np.ndarray) -> torch.Tensor:
        """Copy ``arr`` into a reusable pinned host buffer (grown on demand) and return its view."""
        bufs = self.__dict__.setdefault("_pin_bufs", {})
        n = arr.size
        buf = bufs.get(key)
        if buf is None or buf.numel() < n or buf.dtype != torch.from_numpy(arr[:0].reshape(-1)).dtype:
            buf = torch.empty(max(n, 256), dtype=torch.from_numpy(arr[:0].reshape(-1)).dtype,
                              pin_memory=self.device.type == "cuda")
            bufs[key] = buf
        view = buf[:n].view(arr.shape)
        view.numpy()[...] = arr
        return view

    def _to_dev(self, arr: np.ndarray) -> torch.Tensor:
        return self._pinned(arr).to(self.device, non_blocking=True)

    def _slot_of(self, s: Sequence, pos: int) -> int:
        bs = self.ecfg.block_size
        return s.block_table[pos // bs] * bs + pos % bs

    def _prefill_arrays(self, plan: ScheduledStep):
        """Token ids, positions, KV slots, query starts, last rows, block tables and lengths of a
        prefill step, built per sequence with array slices (no per-token Python work), plus the
        rows / values of image embeddings that replace token embeddings."""
        bs = self.ecfg.block_size
        ids_p, pos_p, slot_p = [], [], []
        e_rows, e_vals = [], []
        q_start = [0]
        total = 0
        for s, n in zip(plan.seqs, plan.n_new):
            c = s.n_cached
            if s.embeds is not None:  # image rows of this chunk
                st, e = s.embeds
                lo, hi = max(st, c), min(st + e.shape[0], c + n)
                if lo < hi:
                    base = total - c
                    e_rows.extend(range(base + lo, base + hi))
                    e_vals.append(e[lo - st: hi - st])
            p = np.arange(c, c + n, dtype=np.int64)
            toks = s.prompt[c:c + n] if c + n <= len(s.prompt) else s.tokens[c:c + n]
            ids_p.append(np.asarray(toks, dtype=np.int32))
            pos_p.append(p)
            tbl = np.asarray(s.block_table, dtype=np.int64)
            slot_p.append(tbl[p // bs] * bs + p % bs)
            total += n
            q_start.append(total)
        S = len(plan.seqs)
        mb = max(len(s.block_table) for s in plan.seqs)
        bt = np.zeros((S, mb), np.int32)
        for i, s in enumerate(plan.seqs):
            bt[i, : len(s.block_table)] = s.block_table
        seq_lens = np.array([s.n_cached + n for s, n in zip(plan.seqs, plan.n_new)], np.int32)
        qs = np.array(q_start, np.int32)
        return (np.concatenate(ids_p), np.concatenate(pos_p).astype(np.int32), np.concatenate(slot_p), qs,
                (qs[1:] - 1).astype(np.int64), bt, seq_lens, e_rows, e_vals)

    def _run_prefill(self, plan: ScheduledStep) -> list[int | None]:
        ids, pos, slots, q_start, last, bt, seq_lens, e_rows, e_vals = self._prefill_arrays(plan)
        inp = StepInput(self._to_dev(ids), self._to_dev(pos), self._to_dev(slots), self._to_dev(bt),
                        self._to_dev(seq_lens), self._to_dev(last), False,
                        q_start=self._to_dev(q_start), max_q=max(plan.n_new))
        if e_rows:
            inp.embed_rows = self._to_dev(np.array(e_rows, np.int64))
            inp.embed_vals = torch.cat(e_vals)
        logits = self.runner.forward(inp)
        complete = [s.n_cached + n >= s.n_tokens for s, n in zip(plan.seqs, plan.n_new)]
        out = self._sample(logits, plan.seqs)
        return [t if c else None for t, c in zip(out, complete)]

    def _decode_arrays(self, seqs: list[Sequence], B: int):
        bs = self.ecfg.block_size
        n = len(seqs)
        ids = np.zeros(B, np.int32)
        pos = np.zeros(B, np.int32)
        slots = np.full(B, self.dummy_block * bs, np.int64)
        lens = np.ones(B, np.int32)
        bt = np.full((B, self.max_blocks_per_seq), self.dummy_block, np.int32)
        for i, s in enumerate(seqs):
            p = s.n_tokens - 1
            ids[i] = s.last_token
            pos[i] = p
            slots[i] = self._slot_of(s, p)
            lens[i] = s.n_tokens
            bt[i, : len(s.block_table)] = s.block_table
        return ids, pos, slots, lens, bt, n

    def _run_decode(self, plan: ScheduledStep) -> list[int | None]:
        seqs = plan.seqs
        simple = all(s.grammar_state is None and s.host_sampler is None and not s.params.needs_penalties
                     and not s.params.logprobs for s in seqs)
        if self.ecfg.cuda_graphs and simple and self.device.type == "cuda":
            B = next((b for b in self.ecfg.graph_buckets if b >= len(seqs)), None)
            if B is not None:
                return self._decode_graph(seqs, B)
        ids, pos, slots, lens, bt, n = self._decode_arrays(seqs, len(seqs))
        inp = StepInput(self._to_dev(ids), self._to_dev(pos), self._to_dev(slots), self._to_dev(bt),
                        self._to_dev(lens), self._to_dev(np.arange(n, dtype=np.int64)), True)
        logits = self.runner.forward(inp)
        return self._sample(logits, seqs)

    # ------------------------------------------------------------------ sampling
    def _sampling_tensors(self, seqs: list[Sequence], B: int):
        temp = np.zeros(B, np.float32)
        topk = np.zeros(B, np.int32)
        topp = np.ones(B, np.float32)
        minp = np.zeros(B, np.float32)
        seeds = np.zeros(B, np.int64)
        steps = np.zeros(B, np.int32)
        for i, s in enumerate(seqs):
            p = s.params
            temp[i] = p.temperature
            topk[i] = p.top_k
            topp[i] = p.top_p
            minp[i] = p.min_p
            seeds[i] = p.seed * 1000003 + s.seq_id if p.seed == 0 else p.seed
            steps[i] = len(s.output)
        return temp, topk, topp, minp, seeds, steps

    def _sample(self, logits: torch.Tensor, seqs: list[Sequence]) -> list[int]:
        B = len(seqs)
        temp, topk, topp, minp, seeds, steps = (self._to_dev(a) for a in self._sampling_tensors(seqs, B))
        mask = None
        if any(s.grammar_state is not None for s in seqs):
            words = (self.cfg.vocab + 31) // 32
            m = np.full((B, words), 0xFFFFFFFF, np.uint32)
            for i, s in enumerate(seqs):
                if s.grammar_state is not None:
                    m[i] = s.grammar_state.allowed_mask(words)
            mask = self._to_dev(m.view(np.int32))
        pen = hist = None
        if any(s.params.needs_penalties for s in seqs):
            nh = max(s.params.penalty_last_n for s in seqs)
            pa = np.zeros((B, 3), np.float32)
            pa[:, 0] = 1.0
            h = np.full((B, nh), -1, np.int32)
            for i, s in enumerate(seqs):
                pa[i] = (s.params.repetition_penalty, s.params.frequency_penalty, s.params.presence_penalty)
                last = s.last_tokens(s.params.penalty_last_n) if s.params.penalty_last_n > 0 else []
                h[i, : len(last)] = last
            pen, hist = self._to_dev(pa), self._to_dev(h)
        host = [i for i, s in enumerate(seqs) if s.host_sampler is not None]
        if host:  # only the rows sampled on the host cross to it
            lg = dict(zip(host, logits[torch.tensor(host, device=logits.device)].float().cpu()))
        ids, _ = ops.sample(logits, temp, topk, topp, minp, seeds, steps, allow_mask=mask, penalties=pen,
                            history=hist)
        out = ids.cpu().tolist()
        for i in host:
            out[i] = seqs[i].host_sampler.sample(lg[i], seqs[i])
        record_logprobs(logits, [i for i, s in enumerate(seqs) if s.params.logprobs], out, seqs)
        return out

    # ------------------------------------------------------------------ CUDA graphs
    def _graph_forward(self, pk: "_Packed"):
        d = pk.d
        inp = StepInput(d["ids"], d["pos"], d["slots"], d["bt"], d["lens"], pk.last, True)
        logits = self.runner.forward(inp)
        ids, _ = ops.sample(logits, d["temp"], d["topk"], d["topp"], d["minp"], d["seeds"], d["steps"])
        return ids

    def _capture(self, B: int) -> _GraphBucket:
        pk = _Packed(B, self.max_blocks_per_seq, self.device)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm up allocations and lazily-set kernel attributes
                self._graph_forward(pk)
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=getattr(self, "_graph_pool", None)):
            out = self._graph_forward(pk)
        self._graph_pool = g.pool()
        gb = _GraphBucket()
        gb.B, gb.graph, gb.out_ids, gb.packed = B, g, out, pk
        return gb

    def _decode_graph(self, seqs: list[Sequence], B: int) -> list[int]:
        gb = self.graphs.get(B)
        if gb is None:
            gb = self.graphs[B] = self._capture(B)
        pk = gb.packed
        n = pk.fill(seqs, self.ecfg.block_size, self.dummy_block)
        pk.upload()  # every per-step input in one host->device copy
        gb.graph.replay()
        return gb.out_ids[:n].cpu().tolist()


class _Packed:
    """Per-step inputs of a B-row decode graph packed into ONE device buffer (and one pinned host
    mirror), so a step uploads everything with a single copy.  Each field is a contiguous typed
    view at a 16-byte aligned offset."""

    FIELDS = (("ids", torch.int32, 0), ("pos", torch.int32, 0), ("lens", torch.int32, 0),
              ("topk", torch.int32, 0), ("steps", torch.int32, 0), ("temp", torch.float32, 0),
              ("topp", torch.float32, 0), ("minp", torch.float32, 0), ("slots", torch.int64, 0),
              ("seeds", torch.int64, 0), ("bt", torch.int32, 1))

    def __init__(self, B: int, max_blocks: int, device):
        lay, off = {}, 0
        for k, dt, is_bt in self.FIELDS:
            n = B * (max_blocks if is_bt else 1) * torch.tensor([], dtype=dt).element_size()
            lay[k] = (off, n, dt, (B, max_blocks) if is_bt else (B,))
            off += (n + 15) // 16 * 16
        self.nbytes = off
        self.dev = torch.zeros(off, dtype=torch.uint8, device=device)
        self.host = torch.zeros(off, dtype=torch.uint8, pin_memory=torch.device(device).type == "cuda")
        self.d = {k: self.dev[o:o + n].view(dt).view(shape) for k, (o, n, dt, shape) in lay.items()}
        self.h = {k: self.host[o:o + n].view(dt).view(shape).numpy() for k, (o, n, dt, shape) in lay.items()}
        self.h["lens"][...] = 1
        self.h["topp"][...] = 1.0
        self.upload()
        self.last = torch.arange(B, dtype=torch.int64, device=device)
        self.B = B
        # what each host row holds: (seq_id, bt_gen, block-table length) or None for a padding row
        self.rows: list = [None] * B
        self.n_prev = B  # rows [n, n_prev) are reset to padding on the next fill

    def fill(self, seqs, block_size: int, dummy: int) -> int:
        """Write a decode step's inputs into the pinned host mirror, touching only what changed: a
        row that holds the same sequence as in this bucket's previous step gets its per-token
        fields and the block-table entries appended since then; a new occupant gets its whole row;
        rows no longer used become padding (dummy page, length 1).  Equal, byte for byte, to
        rewriting every array each step."""
        h, rows, n = self.h, self.rows, len(seqs)
        lens = [s.n_tokens for s in seqs]
        pos = [x - 1 for x in lens]
        h["ids"][:n] = [s.last_token for s in seqs]
        h["pos"][:n] = pos
        h["lens"][:n] = lens
        h["slots"][:n] = [s.block_table[p // block_size] * block_size + p % block_size for s, p in zip(seqs, pos)]
        h["steps"][:n] = [len(s.output) for s in seqs]
        bt = h["bt"]
        for i, s in enumerate(seqs):
            tbl = s.block_table
            nb = len(tbl)
            key = rows[i]
            if key is not None and key[0] == s.seq_id and key[1] == s.bt_gen and key[2] <= nb:
                if nb > key[2]:
                    bt[i, key[2]:nb] = tbl[key[2]:]
            else:
                bt[i, :nb] = tbl
                bt[i, nb:] = dummy
                p = s.params
                h["temp"][i] = p.temperature
                h["topk"][i] = p.top_k
                h["topp"][i] = p.top_p
                h["minp"][i] = p.min_p
                h["seeds"][i] = p.seed * 1000003 + s.seq_id if p.seed == 0 else p.seed
            rows[i] = (s.seq_id, s.bt_gen, nb)
        if self.n_prev > n:
            lo, hi = n, self.n_prev
            for k, v in (("ids", 0), ("pos", 0), ("lens", 1), ("topk", 0), ("steps", 0), ("temp", 0.0),
                         ("topp", 1.0), ("minp", 0.0), ("seeds", 0)):
                h[k][lo:hi] = v
            h["slots"][lo:hi] = dummy * block_size
            bt[lo:hi] = dummy
            for i in range(lo, hi):
                rows[i] = None
        self.n_prev = n
        return n

    def upload(self) -> None:
        self.dev.copy_(self.host, non_blocking=True)


def _attach_health(r, comm, global_rank: int, global_world: int, ec: "EngineConfig") -> None:
    from torch.distributed.distributed_c10d import _get_default_store

    from ..parallel.health import FaultInjector, Heartbeat

    r.injector = FaultInjector(global_rank)
    r.health = Heartbeat(_get_default_store(), global_rank, global_world, timeout=ec.rank_timeout_s,
                         injector=r.injector)


def make_runner(cfg: ModelConfig, tensors, device, kv_dtype, ec: EngineConfig):
    if ec.pp > 1 and ec.tp > 1:
        # tp x pp grid: each pipeline stage is a tensor-parallel group (global rank = stage * tp + t)
        import datetime

        import torch.distributed as dist

        from ..parallel.comm import Comm
        from ..parallel.pp import PPInfo, grid_groups, shard_pp, stage_layers
        from ..parallel.tp import shard_config, shard_tensors

        if not dist.is_initialized():
            dist.init_process_group("nccl", device_id=torch.device(device), timeout=datetime.timedelta(seconds=120))
        stage, t, tp_group, pp_group = grid_groups(ec.tp, ec.pp)
        l0, l1 = stage_layers(cfg.n_layers, ec.pp)[stage]
        comm = Comm(torch.device(device), fused=ec.fused_comm,
                    max_elems=max(ec.max_num_batched_tokens, ec.max_num_seqs) * cfg.hidden, hidden=cfg.hidden,
                    group=tp_group)
        stage_tensors = shard_pp(tensors, cfg.n_layers, stage, ec.pp)
        shard, info = shard_tensors(cfg, stage_tensors, t, ec.tp)
        r = LlamaRunner(shard_config(cfg, ec.tp), shard, device, kv_dtype, act_x2=ec.act_x2, tp=info, comm=comm,
                        pp=PPInfo(stage, ec.pp, l0, l1, tp=ec.tp, tp_rank=t, group=pp_group))
        _attach_health(r, comm, dist.get_rank(), dist.get_world_size(), ec)
        r.ser_threshold = ec.ser_threshold
        r.fused_moe = ec.fused_moe
        dist.barrier()
        return r
    if ec.pp > 1:
        import datetime

        import torch.distributed as dist

        from ..parallel.pp import PPInfo, shard_pp, stage_layers

        if not dist.is_initialized():
            dist.init_process_group("nccl", device_id=torch.device(device), timeout=datetime.timedelta(seconds=120))
        stage, world = dist.get_rank(), dist.get_world_size()
        if world != ec.pp:
            raise ValueError(f"pp={ec.pp} but the process group has {world} ranks")
        l0, l1 = stage_layers(cfg.n_layers, world)[stage]
        r = LlamaRunner(cfg, shard_pp(tensors, cfg.n_layers, stage, world), device, kv_dtype, act_x2=ec.act_x2,
                        pp=PPInfo(stage, world, l0, l1))
        r.ser_threshold = ec.ser_threshold
        r.fused_moe = ec.fused_moe
        dist.barrier()
        return r
    if ec.tp > 1:
        from ..parallel.comm import Comm
        from ..parallel.tp import shard_config, shard_tensors

        comm = Comm(torch.device(device), fused=ec.fused_comm,
                    max_elems=max(ec.max_num_batched_tokens, ec.max_num_seqs) * cfg.hidden, hidden=cfg.hidden,
                    sp_tokens=max(ec.max_num_batched_tokens, ec.max_num_seqs),
                    act_dtype=torch.bfloat16 if cfg.arch.startswith("deepseek") else torch.float16,
                    ep_experts=cfg.n_experts if ec.fused_moe else 0, ep_topk=cfg.n_experts_used)
        if comm.world != ec.tp:
            raise ValueError(f"tp={ec.tp} but the process group has {comm.world} ranks")
        shard, info = shard_tensors(cfg, tensors, comm.rank, comm.world)
        if cfg.is_mla:
            from ..models.deepseek2 import DeepseekV2Runner

            r = DeepseekV2Runner(cfg, shard, device, kv_dtype, ser_threshold=ec.ser_threshold, act_x2=ec.act_x2,
                                 tp=info, comm=comm)
        else:
            r = LlamaRunner(shard_config(cfg, comm.world), shard, device, kv_dtype, act_x2=ec.act_x2, tp=info,
                            comm=comm)
        comm.barrier()  # ranks finish building (tiling) their shards before the first collective
        _attach_health(r, comm, comm.rank, comm.world, ec)
        r.ser_threshold = ec.ser_threshold
        r.fused_moe = ec.fused_moe
        return r
    if cfg.is_mla:
        from ..models.deepseek2 import DeepseekV2Runner

        return DeepseekV2Runner(cfg, tensors, device, kv_dtype, ser_threshold=ec.ser_threshold)
    r = LlamaRunner(cfg, tensors, device, kv_dtype, act_x2=ec.act_x2)
    r.ser_threshold = ec.ser_threshold
    r.fused_moe = ec.fused_moe
    return r


def env_flag(name: str, default: bool) -> bool:
    v = os.environ.get(name)
    return default if v is None else v not in ("0", "false", "False", "")
