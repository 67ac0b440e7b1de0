"""Data parallelism: independent engine replicas, one process per GPU, behind one request front end.

Parity: ``ParallelismStrategy::DataParallel`` / ``MultiGpuConfig::data_parallel``
(``backend/src/cuda_multi_gpu.rs:39,82-90``) — in the reference a configuration value only; nothing
routes requests to replicas.  Here each replica is a full engine (its own weights, KV pool, CUDA
graphs) in its own process pinned to one device, so there is no collective on the hot path; the
front end in the serving process sends each request to one replica and streams its tokens back.

Routing: least outstanding work.  A request costs ``prompt + max_tokens`` tokens when admitted and
its cost falls by one per streamed token, so a replica busy with long generations receives fewer
new requests.  A request whose leading ``affinity_tokens`` prompt tokens were last served by a
replica goes back to that replica while its load is within ``affinity_slack`` tokens of the least
loaded one, so shared prompt prefixes (system prompts) hit that replica's prefix cache.

Failure handling: a replica process that exits (crash, OOM kill) is noticed by the router thread;
its in-flight requests end with ``finish_reason="error"`` and new requests skip it.  A replica whose
``step`` raises fails only the requests it holds and keeps serving.  The front end presents the
``AsyncEngine`` caller API (``stream``, ``generate_blocking``, ``healthy``, ``last_error``,
``shutdown``), so the OpenAI and UDS servers take it unchanged.
"""
from __future__ import annotations

import asyncio
import itertools
import multiprocessing as mp
import os
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable

from ..engine.sampling_params import SamplingParams
from ..server.async_engine import StreamItem

# ------------------------------------------------------------------ engine factories (picklable)


@dataclass
class PresetEngineFactory:
    """Builds a random-init engine of a preset architecture on the replica's device: CPUEngine for
    ``cpu``, the CUDA engine otherwise.  Used by tests and synthetic serving benchmarks."""
    preset: str = "tiny"
    overrides: dict = field(default_factory=dict)
    seed: int = 0
    engine_kw: dict = field(default_factory=dict)

    def __call__(self, device: str):
        from ..models import POLICIES, preset, random_tensors
        from ..models.weights import QuantPolicy
        from ..tokenizer.gguf_tokenizer import synthetic_tokenizer

        cfg = preset(self.preset, **self.overrides)
        t = random_tensors(cfg, POLICIES.get(self.preset, QuantPolicy()), seed=self.seed)
        if device == "cpu":
            from ..engine.cpu_engine import CPUEngine

            eng = CPUEngine(cfg, t, **self.engine_kw)
        else:
            from ..engine.engine import Engine, EngineConfig

            eng = Engine(cfg, t, EngineConfig(device=device, **self.engine_kw))
        eng.tokenizer = synthetic_tokenizer(cfg.vocab)
        return eng


@dataclass
class GGUFEngineFactory:
    """Builds the engine the CLI would build from its parsed arguments (``cli.load``), on the
    replica's device."""
    args: dict

    def __call__(self, device: str):
        import argparse

        from ..cli import load

        a = dict(self.args)
        a.update(device="cpu" if device == "cpu" else "cuda", tp=1, pp=1, dp=1)
        ns = argparse.Namespace(**a)
        if device != "cpu":
            import torch

            torch.cuda.set_device(torch.device(device))
        eng, _, _, _ = load(ns)
        return eng


# ------------------------------------------------------------------ replica process


def _replica_main(idx: int, device: str, factory: Callable[[str], Any], inq, outq, stats_every: float) -> None:
    """Replica loop: admit requests from ``inq``, run engine steps, send the step's token events to
    ``outq`` (this replica's own pipe to the front end) as one message per step.  Messages in: ("req", rid, prompt, params) | ("cancel", rid) |
    ("stop",).  Messages out (tagged with ``idx``): ("ready", info) | ("events", [(rid, tok, reason)])
    with tok None on finish | ("stats", dict) | ("fatal", msg)."""
    if device != "cpu":
        import torch

        torch.cuda.set_device(torch.device(device))
    try:
        eng = factory(device)
        if hasattr(eng, "stop"):  # a multi-rank replica: its follower ranks exit with this process
            import atexit

            atexit.register(eng.stop)
    except Exception as e:  # report and exit; the front end marks the replica dead
        outq.send((idx, "fatal", f"{type(e).__name__}: {e}"))
        return
    outq.send((idx, "ready", {"device": device, "pid": os.getpid()}))
    live: dict[str, Any] = {}
    events: list = []

    def admit(rid, prompt, params):
        def on_token(seq, tok, rid=rid):
            if tok < 0:
                events.append((rid, None, seq.finish_reason or "stop"))
                live.pop(rid, None)
            elif seq.params.logprobs and len(seq.logprobs) >= len(seq.output):
                i = len(seq.output) - 1  # this token's record (the engine records before the callback)
                tops = seq.top_logprobs[i] if i < len(seq.top_logprobs) else []
                events.append((rid, int(tok), None, (float(seq.logprobs[i]), [(int(a), float(v)) for a, v in tops])))
            else:
                events.append((rid, int(tok), None))

        try:
            live[rid] = eng.add_request(prompt, params, rid, on_token=on_token)
        except Exception as e:
            events.append((rid, None, "error:" + str(e)))

    def cancel(rid, reason="abort"):
        seq = live.pop(rid, None)
        if seq is None:
            return
        sched = getattr(eng, "sched", None)
        if sched is not None:
            sched.abort(seq)
        else:
            for lst in (eng.waiting, eng.running):
                if seq in lst:
                    lst.remove(seq)
        events.append((rid, None, reason))

    last_stats = time.monotonic()
    while True:
        block = not eng.has_work() and not events
        try:
            msg = inq.get(timeout=0.05) if block else inq.get_nowait()
            while True:
                if msg[0] == "stop":
                    if events:
                        outq.send((idx, "events", events))
                    if hasattr(eng, "stop"):  # release the follower ranks of a multi-rank replica
                        eng.stop()
                    return
                if msg[0] == "req":
                    admit(msg[1], msg[2], msg[3])
                elif msg[0] == "cancel":
                    cancel(msg[1])
                msg = inq.get_nowait()
        except queue.Empty:
            pass
        if eng.has_work():
            try:
                eng.step()
            except Exception as e:  # fail what this replica holds, keep serving
                err = f"error:{type(e).__name__}: {e}"
                for rid in list(live):
                    cancel(rid, err)
                sched = getattr(eng, "sched", None)
                if sched is not None:
                    sched.clear_waiting("error")
        if events:
            outq.send((idx, "events", events))
            events = []
        now = time.monotonic()
        if now - last_stats >= stats_every:
            last_stats = now
            t = dict(getattr(eng, "timings", {}) or {})
            blocks = getattr(eng, "blocks", None)
            if blocks is not None:
                t["kv_blocks_used"], t["kv_blocks_total"] = blocks.n_used, blocks.num_blocks
            t["in_flight"] = len(live)
            outq.send((idx, "stats", t))


# ------------------------------------------------------------------ front end


@dataclass
class _Request:
    rid: str
    replica: int
    cost: int
    sink: "queue.Queue[StreamItem] | None" = None
    loop: asyncio.AbstractEventLoop | None = None
    aqueue: asyncio.Queue | None = None
    lp: Any = None  # _LogprobRecord of a request that asked for logprobs


class _LogprobRecord:
    """Front-end copy of a replica sequence's per-token log-probabilities, passed as ``StreamItem.seq``
    so that the servers read them as they read a local engine's sequence."""

    def __init__(self):
        self.logprobs: list[float] = []
        self.top_logprobs: list[list[tuple[int, float]]] = []


@dataclass
class ReplicaState:
    idx: int
    device: str
    proc: Any = None
    inq: Any = None
    alive: bool = False
    load: int = 0  # outstanding tokens (prompt + remaining max_tokens) of its in-flight requests
    served: int = 0
    stats: dict = field(default_factory=dict)
    error: str | None = None
    out: Any = None  # read end of the replica's pipe (None once it has closed)


class DataParallelEngine:
    """``n`` engine replicas on ``devices`` (default ``cuda:0..n-1``; ``cpu`` entries run CPUEngine
    replicas), each built in its own process by ``factory(device)``."""

    def __init__(self, factory: Callable[[str], Any], devices: list[str], cfg=None, tokenizer=None,
                 affinity_tokens: int = 32, affinity_slack: int = 512, start_timeout: float = 600.0,
                 stats_every: float = 1.0):
        if not devices:
            raise ValueError("data parallelism needs at least one replica device")
        self.cfg = cfg
        self.tokenizer = tokenizer
        self.affinity_tokens = affinity_tokens
        self.affinity_slack = affinity_slack
        ctx = mp.get_context("spawn")
        self.replicas = [ReplicaState(i, d) for i, d in enumerate(devices)]
        for r in self.replicas:
            r.inq = ctx.Queue()
            # one pipe per replica to the front end, written by that replica only: a replica killed
            # in the middle of a send can only break its own pipe (a queue shared by all replicas
            # keeps a cross-process write lock that a killed writer can leave held, which would
            # silence every survivor)
            r.out, out_w = ctx.Pipe(duplex=False)
            # not daemonic: a replica may start processes of its own (the other ranks of a
            # multi-GPU replica); shutdown() stops and joins every replica
            r.proc = ctx.Process(target=_replica_main, args=(r.idx, r.device, factory, r.inq, out_w, stats_every),
                                 name=f"barq-dp{r.idx}", daemon=False)
            r.proc.start()
            out_w.close()  # the replica holds the only write end: its exit shows up as EOF here
        self._lock = threading.Lock()
        self._reqs: dict[str, _Request] = {}
        self._affinity: dict[tuple, int] = {}
        self._ids = itertools.count()
        self._stop = threading.Event()
        self.last_error: str | None = None
        import atexit

        atexit.register(self.shutdown)  # replica processes are not daemonic: stop them at exit
        self._wait_ready(start_timeout)
        self._router = threading.Thread(target=self._route_loop, name="barq-dp-router", daemon=True)
        self._router.start()

    # ------------------------------------------------------------------ lifecycle
    def _recv(self, timeout: float) -> list[tuple]:
        """Messages that arrive on any replica pipe within ``timeout`` s; a pipe that closes or
        breaks (its replica exited, possibly mid-message) yields a ("fatal", why) message once."""
        from multiprocessing.connection import wait

        conns = {r.out: r for r in self.replicas if r.out is not None}
        if not conns:
            time.sleep(timeout)
            return []
        msgs = []
        for c in wait(list(conns), timeout):
            r = conns[c]
            try:
                while True:
                    msgs.append(c.recv())
                    if not c.poll():
                        break
            except (EOFError, OSError) as e:
                r.out = None
                c.close()
                code = r.proc.exitcode if r.proc is not None else None
                msgs.append((r.idx, "fatal", f"replica {r.idx} ({r.device}) exited with code {code}"
                             if isinstance(e, EOFError) else f"replica {r.idx} pipe broke: {e}"))
            except Exception as e:  # a partial message from a replica killed mid-send
                r.out = None
                c.close()
                msgs.append((r.idx, "fatal", f"replica {r.idx} sent a broken message: {type(e).__name__}"))
        return msgs

    def _wait_ready(self, timeout: float) -> None:
        pending = {r.idx for r in self.replicas}
        deadline = time.monotonic() + timeout
        while pending:
            left = deadline - time.monotonic()
            if left <= 0:
                self.shutdown()
                raise TimeoutError(f"data-parallel replicas {sorted(pending)} not ready after {timeout:.0f} s")
            for idx, kind, payload in self._recv(min(left, 1.0)):
                r = self.replicas[idx]
                if kind == "ready":
                    r.alive = True
                elif kind == "fatal":
                    r.error = payload
                pending.discard(idx)
        if not any(r.alive for r in self.replicas):
            errs = "; ".join(f"{r.idx}: {r.error}" for r in self.replicas)
            self.shutdown()
            raise RuntimeError(f"no data-parallel replica started ({errs})")

    def shutdown(self) -> None:
        self._stop.set()
        for r in self.replicas:
            if r.proc is not None and r.proc.is_alive():
                try:
                    r.inq.put(("stop",))
                except Exception:
                    pass
        for r in self.replicas:
            if r.proc is not None:
                r.proc.join(timeout=10)
                if r.proc.is_alive():
                    r.proc.terminate()
                    r.proc.join(timeout=5)
            r.alive = False
        router = getattr(self, "_router", None)
        if router is not None and router is not threading.current_thread():
            router.join(timeout=5)

    @property
    def healthy(self) -> bool:
        return any(r.alive for r in self.replicas)

    @property
    def n_alive(self) -> int:
        return sum(r.alive for r in self.replicas)

    @property
    def timings(self) -> dict:
        """Replica engine timings summed over live replicas (as last reported)."""
        out: dict = {}
        for r in self.replicas:
            for k, v in r.stats.items():
                if isinstance(v, (int, float)):
                    out[k] = out.get(k, 0) + v
        return out

    # ------------------------------------------------------------------ routing
    def _pick(self, prompt: list[int], cost: int) -> int:
        live = [r for r in self.replicas if r.alive]
        if not live:
            raise RuntimeError("no live data-parallel replica" + (f" ({self.last_error})" if self.last_error else ""))
        best = min(live, key=lambda r: (r.load, r.served))
        if self.affinity_tokens > 0 and len(prompt) >= self.affinity_tokens:
            key = tuple(prompt[: self.affinity_tokens])
            i = self._affinity.get(key)
            if i is not None and self.replicas[i].alive and self.replicas[i].load <= best.load + self.affinity_slack:
                best = self.replicas[i]
            self._affinity[key] = best.idx
            if len(self._affinity) > 65536:  # bounded: forget the oldest half
                for k in list(self._affinity)[:32768]:
                    del self._affinity[k]
        return best.idx

    def _submit(self, prompt: list[int], params: SamplingParams, request_id: str, **sink) -> _Request:
        rid = f"{request_id or 'req'}#{next(self._ids)}"
        cost = len(prompt) + int(params.max_tokens)
        with self._lock:
            idx = self._pick(prompt, cost)
            req = _Request(rid, idx, cost, **sink)
            self._reqs[rid] = req
            r = self.replicas[idx]
            r.load += cost
            r.served += 1
        r.inq.put(("req", rid, list(prompt), params))
        return req

    def _deliver(self, req: _Request, item: StreamItem) -> None:
        if req.aqueue is not None and req.loop is not None:
            req.loop.call_soon_threadsafe(req.aqueue.put_nowait, item)
        elif req.sink is not None:
            req.sink.put(item)

    def _end(self, rid: str, reason: str) -> None:
        with self._lock:
            req = self._reqs.pop(rid, None)
            if req is None:
                return
            r = self.replicas[req.replica]
            r.load -= req.cost
        self._deliver(req, StreamItem(None, reason))

    def _route_loop(self) -> None:
        last_check = time.monotonic()
        while not self._stop.is_set():
            for idx, kind, payload in self._recv(0.05):
                if kind == "events":
                    for rid, tok, reason, *lp in payload:
                        if tok is None:
                            self._end(rid, reason)
                            continue
                        with self._lock:
                            req = self._reqs.get(rid)
                            if req is not None and req.cost > 0:
                                req.cost -= 1
                                self.replicas[req.replica].load -= 1
                        if req is not None:
                            if lp:
                                if req.lp is None:
                                    req.lp = _LogprobRecord()
                                req.lp.logprobs.append(lp[0][0])
                                req.lp.top_logprobs.append(lp[0][1])
                            self._deliver(req, StreamItem(tok, None, req.lp))
                elif kind == "stats":
                    self.replicas[idx].stats = payload
                elif kind == "fatal":
                    self._mark_dead(idx, payload)
            now = time.monotonic()
            if now - last_check > 0.2:
                last_check = now
                for r in self.replicas:
                    if r.alive and not r.proc.is_alive():
                        self._mark_dead(r.idx, f"replica {r.idx} ({r.device}) exited with code {r.proc.exitcode}")

    def _mark_dead(self, idx: int, msg: str) -> None:
        r = self.replicas[idx]
        r.alive = False
        r.error = msg
        self.last_error = msg
        with self._lock:
            rids = [rid for rid, q in self._reqs.items() if q.replica == idx]
        for rid in rids:
            self._end(rid, "error:" + msg)

    # ------------------------------------------------------------------ caller side (AsyncEngine API)
    @staticmethod
    def _check(item: StreamItem) -> StreamItem:
        if item.token is None and item.finish_reason and item.finish_reason.startswith("error"):
            raise ValueError(item.finish_reason[6:] or "replica error")
        return item

    async def stream(self, prompt: list[int], params: SamplingParams, request_id: str = ""):
        """Async generator of StreamItem; the last item has token None."""
        loop = asyncio.get_running_loop()
        req = self._submit(prompt, params, request_id, loop=loop, aqueue=asyncio.Queue())
        done = False
        try:
            while True:
                item = await req.aqueue.get()
                done = item.token is None
                yield self._check(item)
                if done:
                    return
        finally:
            if not done:  # the consumer went away: the replica stops generating for it
                self.cancel(req.rid)

    def cancel(self, rid: str) -> None:
        with self._lock:
            req = self._reqs.pop(rid, None)
            if req is None:
                return
            r = self.replicas[req.replica]
            r.load -= req.cost
        if r.alive:
            r.inq.put(("cancel", rid))

    def generate_blocking(self, prompt: list[int], params: SamplingParams, request_id: str = "", timeout=None):
        """Iterator of StreamItem for synchronous callers (UDS server, CLI)."""
        req = self._submit(prompt, params, request_id, sink=queue.Queue())
        done = False
        try:
            while True:
                item = req.sink.get(timeout=timeout)
                done = item.token is None
                yield self._check(item)
                if done:
                    return
        finally:
            if not done:  # the caller closed the iterator early: the replica stops generating for it
                self.cancel(req.rid)

    def generate(self, prompts: list[list[int]], params: SamplingParams | None = None) -> list[list[int]]:
        """Runs every prompt to completion across the replicas; returns the token lists in order."""
        params = params or SamplingParams()
        reqs = [self._submit(p, params, f"batch{i}", sink=queue.Queue()) for i, p in enumerate(prompts)]
        outs = []
        for req in reqs:
            toks = []
            while True:
                item = self._check(req.sink.get())
                if item.token is None:
                    break
                toks.append(item.token)
            outs.append(toks)
        return outs

    def replica_info(self) -> list[dict]:
        return [{"replica": r.idx, "device": r.device, "alive": r.alive, "load": r.load, "served": r.served,
                 "error": r.error} for r in self.replicas]


def default_devices(n: int) -> list[str]:
    """``cuda:0..n-1`` when that many GPUs are visible, else ``cpu`` replicas."""
    try:
        import torch

        if torch.cuda.is_available() and torch.cuda.device_count() >= n:
            return [f"cuda:{i}" for i in range(n)]
    except Exception:
        pass
    return ["cpu"] * n


# ------------------------------------------------------------------ replicas that span several GPUs


def _tp_follower(rank: int, tp: int, port: int, backend: str, device: str, builder) -> None:
    import torch.distributed as dist

    from .lockstep import follower_loop

    if device != "cpu":
        import torch

        torch.cuda.set_device(torch.device(device))
    dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=tp)
    eng = builder(device, rank, tp)
    from torch.distributed.distributed_c10d import _get_default_store

    follower_loop(eng, _get_default_store())


def _free_port() -> int:
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@dataclass
class TPReplicaFactory:
    """A data-parallel replica that is itself a tensor-parallel group of ``tp`` ranks: the replica
    process becomes rank 0 (wrapped in a ``LockstepLeader``) and starts ranks 1..tp-1, which replay
    its steps.  ``builder(device, rank, world)`` returns one rank's engine after the process group
    is up (``GGUFTPBuilder`` for a GGUF file).  A replica given ``cuda:k`` uses GPUs k..k+tp-1."""
    builder: Callable
    tp: int

    def __call__(self, device: str):
        import torch.distributed as dist
        from torch.distributed.distributed_c10d import _get_default_store

        from .lockstep import LockstepLeader

        backend = "gloo" if device == "cpu" else "nccl"
        base = 0 if device == "cpu" else int(device.split(":")[1])
        devs = ["cpu"] * self.tp if device == "cpu" else [f"cuda:{base + i}" for i in range(self.tp)]
        port = _free_port()
        ctx = mp.get_context("spawn")
        self.procs = [ctx.Process(target=_tp_follower, args=(i, self.tp, port, backend, devs[i], self.builder),
                                  daemon=True) for i in range(1, self.tp)]
        for p in self.procs:
            p.start()
        dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=self.tp)
        eng = self.builder(devs[0], 0, self.tp)
        return LockstepLeader(eng, _get_default_store())


@dataclass
class GGUFTPBuilder:
    """One rank of a tensor-parallel engine built from CLI arguments (``cli.load`` with ``--tp``)."""
    args: dict

    def __call__(self, device: str, rank: int, world: int):
        import argparse
        import os as _os

        from ..cli import load

        _os.environ["LOCAL_RANK"] = device.split(":")[1] if ":" in device else "0"
        a = dict(self.args)
        a.update(device="cuda", tp=world, pp=1, dp=1)
        eng, _, _, _ = load(argparse.Namespace(**a))
        return eng
