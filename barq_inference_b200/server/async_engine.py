"""Thread-safe streaming front for an engine: one background thread owns the engine and runs
continuous-batching steps; callers submit requests and consume tokens as they are sampled.

Parity: ``BatchEngine`` / ``BatchEngineHandle::submit`` (``advanced/src/batch_engine.rs:45-191``, an
mpsc request queue drained by a tokio loop) — but the forward pass here is the real batched model,
so every request in flight shares each decode step, and tokens are streamed per step (the
reference's HTTP server generates the whole completion before it starts streaming,
``cli/src/server.rs:738``).
"""
from __future__ import annotations

import asyncio
import queue
import threading
import time
from dataclasses import dataclass, field

from ..engine.sampling_params import SamplingParams


@dataclass
class StreamItem:
    token: int | None  # None = finished
    finish_reason: str | None = None
    seq: object = None


@dataclass
class Submission:
    prompt: list[int]
    params: SamplingParams
    request_id: str
    sink: "queue.Queue[StreamItem] | None" = None
    loop: asyncio.AbstractEventLoop | None = None
    aqueue: asyncio.Queue | None = None
    error: list = field(default_factory=list)
    accepted: threading.Event = field(default_factory=threading.Event)


def _refusal(e: Exception) -> Exception:
    """What the caller sees for a request the engine did not accept: admission-control refusals
    keep their type (servers answer 503), anything else is a bad request (ValueError)."""
    from ..engine.scheduler import Overloaded

    return e if isinstance(e, Overloaded) else ValueError(str(e))


@dataclass
class _Call:
    """A function to run on the engine thread between steps (e.g. embeddings)."""
    fn: object
    done: threading.Event = field(default_factory=threading.Event)
    result: object = None
    error: BaseException | None = None


class AsyncEngine:
    def __init__(self, engine, metrics=None, idle_sleep: float = 0.002):
        self.engine = engine
        self.metrics = metrics
        self.inbox: "queue.Queue[Submission]" = queue.Queue()
        self.idle_sleep = idle_sleep
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="barq-engine", daemon=True)
        self._thread.start()
        self.healthy = True
        self.last_error: str | None = None

    def shutdown(self) -> None:
        self._stop.set()
        self._thread.join(timeout=5)

    # ------------------------------------------------------------------ engine thread
    def _deliver(self, sub: Submission, item: StreamItem) -> None:
        if sub.aqueue is not None and sub.loop is not None:
            try:
                sub.loop.call_soon_threadsafe(sub.aqueue.put_nowait, item)
            except RuntimeError:  # the consumer's event loop is gone; its abort is on the way
                pass
        elif sub.sink is not None:
            sub.sink.put(item)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                while True:
                    sub = self.inbox.get_nowait()
                    if isinstance(sub, _Call):
                        try:
                            sub.result = sub.fn(self.engine)
                        except BaseException as e:  # noqa: BLE001 - handed to the caller
                            sub.error = e
                        sub.done.set()
                    else:
                        self._admit(sub)
            except queue.Empty:
                pass
            if not self.engine.has_work():
                time.sleep(self.idle_sleep)
                continue
            try:
                self.engine.step()
                self.healthy = True
            except Exception as e:  # fail the in-flight requests, keep serving
                self.healthy = False
                self.last_error = f"{type(e).__name__}: {e}"
                self._fail_all(self.last_error)

    def _admit(self, sub: Submission) -> None:
        def on_token(seq, tok, sub=sub):
            if tok < 0:
                self._deliver(sub, StreamItem(None, seq.finish_reason, seq))
            else:
                self._deliver(sub, StreamItem(tok, None, seq))

        try:
            seq = self.engine.add_request(sub.prompt, sub.params, sub.request_id, on_token=on_token)
            sub.seq = seq
        except Exception as e:
            sub.error.append(e)
            self._deliver(sub, StreamItem(None, "error"))
        sub.accepted.set()

    def _fail_all(self, msg: str) -> None:
        eng = self.engine
        seqs = list(getattr(getattr(eng, "sched", None), "running", [])) + list(getattr(getattr(eng, "sched", None), "waiting", []))
        seqs += list(getattr(eng, "running", [])) + list(getattr(eng, "waiting", []))
        for s in seqs:
            s.finish_reason = "error"
            if s.on_token is not None:
                s.on_token(s, -1)
        if hasattr(eng, "sched"):
            for s in list(eng.sched.running):
                eng.sched.finish(s, "error")
            eng.sched.clear_waiting("error")
        else:
            eng.running.clear()
            eng.waiting.clear()

    # ------------------------------------------------------------------ caller side
    async def stream(self, prompt: list[int], params: SamplingParams, request_id: str = ""):
        """Async generator of StreamItem; the last item has token None."""
        loop = asyncio.get_running_loop()
        sub = Submission(prompt, params, request_id, loop=loop, aqueue=asyncio.Queue())
        self.inbox.put(sub)
        done = False
        try:
            while True:
                item = await sub.aqueue.get()
                done = item.token is None  # before the yield: a consumer may stop right after the last item
                if done and item.finish_reason == "error" and sub.error:
                    raise _refusal(sub.error[0])
                yield item
                if done:
                    return
        finally:
            if not done:  # the consumer stopped early (client disconnected): stop generating for it
                self._abort(sub)

    def _abort(self, sub: Submission) -> None:
        def fn(eng, sub=sub):
            seq = getattr(sub, "seq", None)
            if seq is not None and hasattr(eng, "abort"):
                eng.abort(seq)

        self.inbox.put(_Call(fn))

    def call_sync(self, fn, timeout: float | None = None):
        """Run ``fn(engine)`` on the engine thread (between steps) and return its result."""
        c = _Call(fn)
        self.inbox.put(c)
        if not c.done.wait(timeout):
            raise TimeoutError("engine call timed out")
        if c.error is not None:
            raise c.error
        return c.result

    async def call(self, fn):
        """Async form of ``call_sync``."""
        loop = asyncio.get_running_loop()
        return await loop.run_in_executor(None, self.call_sync, fn)

    def generate_blocking(self, prompt: list[int], params: SamplingParams, request_id: str = "", timeout=None):
        """Iterator of StreamItem for synchronous callers (UDS server, CLI)."""
        sub = Submission(prompt, params, request_id, sink=queue.Queue())
        self.inbox.put(sub)
        done = False
        try:
            while True:
                item = sub.sink.get(timeout=timeout)
                done = item.token is None  # before the yield: a caller may stop right after the last item
                if done and item.finish_reason == "error" and sub.error:
                    raise _refusal(sub.error[0])
                yield item
                if done:
                    return
        finally:
            if not done:  # the caller stopped early (closed the iterator): stop generating for it
                self._abort(sub)
