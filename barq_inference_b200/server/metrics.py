"""Inference metrics with a Prometheus text exporter, request guards and context health.

Parity: ``InferenceMetrics`` / ``RequestGuard`` / ``ContextManager`` (``advanced/src/metrics.rs:14-340``)
and the Prometheus exporter of ``advanced/src/metrics_server.rs:179-215`` (compiled out in the
reference, ``advanced/src/lib.rs:50``).  Metric names keep the reference's ``barq_*`` prefix.
"""
from __future__ import annotations

import bisect
import enum
import threading
import time

TTFT_BUCKETS = (0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1.0, 2.5, 5.0, 10.0)
TPOT_BUCKETS = (0.001, 0.002, 0.005, 0.01, 0.02, 0.05, 0.1, 0.25, 0.5, 1.0)


class _Hist:
    def __init__(self, buckets):
        self.b = tuple(buckets)
        self.counts = [0] * (len(self.b) + 1)
        self.sum = 0.0
        self.n = 0

    def observe(self, v: float) -> None:
        self.counts[bisect.bisect_left(self.b, v)] += 1
        self.sum += v
        self.n += 1

    def lines(self, name: str) -> list[str]:
        out, acc = [], 0
        for le, c in zip(self.b, self.counts):
            acc += c
            out.append(f'{name}_bucket{{le="{le}"}} {acc}')
        out.append(f'{name}_bucket{{le="+Inf"}} {self.n}')
        out.append(f"{name}_sum {self.sum}")
        out.append(f"{name}_count {self.n}")
        return out


class InferenceMetrics:
    def __init__(self):
        self._lock = threading.Lock()
        self.requests_total = 0
        self.requests_successful = 0
        self.requests_failed = 0
        self.requests_active = 0
        self.requests_peak_concurrent = 0
        self.tokens_generated = 0
        self.prompt_tokens = 0
        self.inference_ms = 0.0
        self.rate_limited = 0
        self.comm_timeouts = 0
        self.ttft = _Hist(TTFT_BUCKETS)
        self.tpot = _Hist(TPOT_BUCKETS)
        self.started = time.time()

    def begin(self) -> "RequestGuard":
        with self._lock:
            self.requests_total += 1
            self.requests_active += 1
            self.requests_peak_concurrent = max(self.requests_peak_concurrent, self.requests_active)
        return RequestGuard(self)

    def _end(self, ok: bool, prompt_tokens: int, gen_tokens: int, elapsed_s: float, ttft_s: float | None):
        with self._lock:
            self.requests_active -= 1
            if ok:
                self.requests_successful += 1
            else:
                self.requests_failed += 1
            self.prompt_tokens += prompt_tokens
            self.tokens_generated += gen_tokens
            self.inference_ms += elapsed_s * 1e3
            if ttft_s is not None:
                self.ttft.observe(ttft_s)
                if gen_tokens > 1:
                    self.tpot.observe((elapsed_s - ttft_s) / (gen_tokens - 1))

    def snapshot(self) -> dict:
        with self._lock:
            done = self.requests_successful + self.requests_failed
            return {
                "requests_total": self.requests_total,
                "requests_successful": self.requests_successful,
                "requests_failed": self.requests_failed,
                "requests_active": self.requests_active,
                "requests_peak_concurrent": self.requests_peak_concurrent,
                "tokens_generated": self.tokens_generated,
                "prompt_tokens": self.prompt_tokens,
                "avg_inference_ms": self.inference_ms / done if done else 0.0,
                "tokens_per_second": self.tokens_generated / max(1e-9, self.inference_ms / 1e3) if done else 0.0,
                "uptime_s": time.time() - self.started,
            }

    def prometheus(self, engine=None) -> str:
        s = self.snapshot()
        lines = []

        def g(name, v, kind="counter", help_=""):
            lines.append(f"# HELP {name} {help_ or name}")
            lines.append(f"# TYPE {name} {kind}")
            lines.append(f"{name} {v}")

        g("barq_requests_total", s["requests_total"], help_="Requests received")
        g("barq_requests_successful", s["requests_successful"])
        g("barq_requests_failed", s["requests_failed"])
        g("barq_requests_active", s["requests_active"], "gauge")
        g("barq_requests_peak_concurrent", s["requests_peak_concurrent"], "gauge")
        g("barq_tokens_generated_total", s["tokens_generated"])
        g("barq_prompt_tokens_total", s["prompt_tokens"])
        g("barq_rate_limited_total", self.rate_limited)
        g("barq_comm_timeouts_total", self.comm_timeouts)
        if engine is not None:
            t = getattr(engine, "timings", {})
            g("barq_prefill_tokens_total", t.get("prefill_tokens", 0))
            g("barq_decode_tokens_total", t.get("decode_tokens", 0))
            blocks = getattr(engine, "blocks", None)
            if blocks is not None:
                g("barq_kv_blocks_used", blocks.n_used, "gauge")
                g("barq_kv_blocks_total", blocks.num_blocks, "gauge")
            spec = getattr(engine, "spec_stats", None)
            if spec is not None:
                g("barq_spec_acceptance_rate", spec.acceptance_rate, "gauge")
            load = getattr(getattr(engine, "runner", None), "expert_load", None) or getattr(
                getattr(engine, "model", None), "expert_load", None)
            if load is not None:  # MoE expert-load counters (BARQ_MOE_STATS=1)
                ms = load.summary()
                g("barq_moe_tokens_routed_total", ms["tokens_routed"])
                g("barq_moe_load_max_over_mean", ms["max_over_mean"], "gauge")
                g("barq_moe_load_cv", ms["cv"], "gauge")
        lines.append("# TYPE barq_ttft_seconds histogram")
        lines += self.ttft.lines("barq_ttft_seconds")
        lines.append("# TYPE barq_tpot_seconds histogram")
        lines += self.tpot.lines("barq_tpot_seconds")
        return "\n".join(lines) + "\n"


class RequestGuard:
    """Marks the request failed unless ``complete`` is called (``metrics.rs:123-152``)."""

    def __init__(self, m: InferenceMetrics):
        self.m = m
        self.t0 = time.perf_counter()
        self.ttft: float | None = None
        self.done = False

    def first_token(self):
        if self.ttft is None:
            self.ttft = time.perf_counter() - self.t0

    def complete(self, prompt_tokens: int, gen_tokens: int):
        if not self.done:
            self.done = True
            self.m._end(True, prompt_tokens, gen_tokens, time.perf_counter() - self.t0, self.ttft)

    def fail(self):
        if not self.done:
            self.done = True
            self.m._end(False, 0, 0, time.perf_counter() - self.t0, None)

    def __enter__(self):
        return self

    def __exit__(self, exc_type, exc, tb):
        if not self.done:
            self.fail()
        return False


class ContextHealth(enum.Enum):
    HEALTHY = "healthy"
    WARNING = "warning"
    CRITICAL = "critical"


def context_health(used_fraction: float, warn: float = 0.8, critical: float = 0.95) -> ContextHealth:
    """KV-pool health thresholds (``metrics.rs:236-340``)."""
    if used_fraction >= critical:
        return ContextHealth.CRITICAL
    if used_fraction >= warn:
        return ContextHealth.WARNING
    return ContextHealth.HEALTHY
