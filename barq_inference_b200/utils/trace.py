"""Step tracing: NVTX ranges and per-step JSON timings.

Parity: the reference has ``tracing`` log macros and a ``BenchmarkTimer``
(``cli/src/main.rs:300-305``, ``barq_core/src/testing.rs:150-182``) but no GPU timers or ranges.

* ``BARQ_NVTX=1``: every engine step (and every layer of the runner's forward) is an NVTX range,
  visible in Nsight Systems timelines.
* ``BARQ_PROFILE=1``: one JSON line per engine step -- step index, kind (prefill/decode), tokens,
  host wall time and device time (CUDA events around the step, resolved one step later so that no
  extra synchronization is added) -- appended to ``BARQ_PROFILE_FILE`` (default: stderr).
"""
from __future__ import annotations

import contextlib
import json
import os
import sys
import time

import torch


def nvtx_enabled() -> bool:
    return os.environ.get("BARQ_NVTX", "0") not in ("0", "", "false")


@contextlib.contextmanager
def nvtx(name: str, enabled: bool | None = None):
    on = nvtx_enabled() if enabled is None else enabled
    if on:
        torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        if on:
            torch.cuda.nvtx.range_pop()


class StepProfiler:
    def __init__(self, engine, path: str | None = None, nvtx_ranges: bool | None = None):
        self.engine = engine
        self.path = path or os.environ.get("BARQ_PROFILE_FILE")
        self.nvtx = nvtx_enabled() if nvtx_ranges is None else nvtx_ranges
        self._pending = None
        self.records: list[dict] = []

    @classmethod
    def from_env(cls, engine):
        if os.environ.get("BARQ_PROFILE", "0") in ("0", "", "false") and not nvtx_enabled():
            return None
        return cls(engine)

    def _emit(self, rec: dict) -> None:
        self.records.append(rec)
        if os.environ.get("BARQ_PROFILE", "0") in ("0", "", "false"):
            return
        line = json.dumps(rec)
        if self.path:
            with open(self.path, "a") as f:
                f.write(line + "\n")
        else:
            print(line, file=sys.stderr, flush=True)

    def _resolve(self) -> None:
        if self._pending is None:
            return
        rec, e0, e1 = self._pending
        if e1 is not None:
            e1.synchronize()
            rec["gpu_ms"] = round(e0.elapsed_time(e1), 4)
        self._emit(rec)
        self._pending = None

    def step(self, fn):
        eng = self.engine
        cuda = eng.device.type == "cuda"
        idx = eng.step_count
        e0 = e1 = None
        if cuda:
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
        t0 = time.perf_counter()
        with nvtx(f"barq.step {idx}", self.nvtx):
            done = fn()
        wall = time.perf_counter() - t0
        if cuda:
            e1 = torch.cuda.Event(enable_timing=True)
            e1.record()
        self._resolve()
        plan = getattr(eng, "last_plan", None)
        rec = {"step": idx, "kind": getattr(plan, "kind", None),
               "tokens": int(sum(plan.n_new)) if plan is not None else 0, "wall_ms": round(wall * 1e3, 4)}
        self._pending = (rec, e0, e1)
        return done

    def flush(self) -> None:
        self._resolve()
