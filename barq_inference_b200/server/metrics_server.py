"""Standalone metrics / health HTTP endpoint (default ``0.0.0.0:9090``) for serving modes without an
HTTP front end of their own (the UDS server), or for scraping on a separate port.

Parity: ``MetricsServer`` / ``MetricsServerConfig`` (``advanced/src/metrics_server.rs:19-184``, a module
the reference leaves disabled): ``GET /metrics``, ``GET /health``, ``GET /``, 404 otherwise.  The
reference answers ``/metrics`` with a JSON snapshot; here ``/metrics`` is the Prometheus text format
(``barq_requests_*`` names, the format scrapers expect) and ``/metrics.json`` is the JSON snapshot.
Runs on the standard library's threaded HTTP server in a daemon thread.
"""
from __future__ import annotations

import json
import threading
import time
from dataclasses import dataclass
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from .metrics import InferenceMetrics, context_health


@dataclass
class MetricsServerConfig:
    host: str = "0.0.0.0"
    port: int = 9090
    metrics_path: str = "/metrics"
    health_path: str = "/health"


class MetricsServer:
    def __init__(self, metrics: InferenceMetrics, config: MetricsServerConfig | None = None, engine=None,
                 health_fn=None):
        """``engine``: adds its KV / timing gauges to the exposition; ``health_fn() -> (ok, detail)``
        overrides the health verdict (e.g. an ``AsyncEngine``'s ``healthy`` flag)."""
        self.metrics = metrics
        self.cfg = config or MetricsServerConfig()
        self.engine = engine
        self.health_fn = health_fn
        self.started = time.time()
        self._httpd = None

    def _health(self) -> tuple[int, dict]:
        blocks = getattr(self.engine, "blocks", None)
        used = blocks.n_used / blocks.num_blocks if blocks is not None else 0.0
        ok, detail = (True, None) if self.health_fn is None else self.health_fn()
        body = {"status": "healthy" if ok else "degraded", "uptime_s": round(time.time() - self.started, 3),
                "kv_usage": used, "context_health": context_health(used).value,
                "metrics": self.metrics.snapshot()}
        if detail:
            body["detail"] = detail
        return (200 if ok else 503), body

    def start(self) -> "MetricsServer":
        srv = self

        class Handler(BaseHTTPRequestHandler):
            def _send(self, code: int, body: str, ctype: str):
                data = body.encode("utf-8")
                self.send_response(code)
                self.send_header("Content-Type", ctype)
                self.send_header("Content-Length", str(len(data)))
                self.end_headers()
                self.wfile.write(data)

            def do_GET(self):  # noqa: N802 (http.server naming)
                path = self.path.split("?", 1)[0]
                if path == srv.cfg.metrics_path:
                    self._send(200, srv.metrics.prometheus(srv.engine), "text/plain; version=0.0.4")
                elif path == srv.cfg.metrics_path + ".json":
                    self._send(200, json.dumps(srv.metrics.snapshot(), indent=2), "application/json")
                elif path == srv.cfg.health_path:
                    code, body = srv._health()
                    self._send(code, json.dumps(body, indent=2), "application/json")
                elif path == "/":
                    self._send(200, json.dumps({"service": "barq-inference metrics",
                                                "endpoints": [srv.cfg.metrics_path, srv.cfg.metrics_path + ".json",
                                                              srv.cfg.health_path]}), "application/json")
                else:
                    self._send(404, json.dumps({"error": "not found"}), "application/json")

            def log_message(self, fmt, *args):  # quiet: request logs go through the barq logger
                pass

        self._httpd = ThreadingHTTPServer((self.cfg.host, self.cfg.port), Handler)
        self._httpd.daemon_threads = True
        threading.Thread(target=self._httpd.serve_forever, name="barq-metrics", daemon=True).start()
        return self

    @property
    def port(self) -> int:
        return self._httpd.server_address[1] if self._httpd is not None else self.cfg.port

    def stop(self) -> None:
        if self._httpd is not None:
            self._httpd.shutdown()
            self._httpd.server_close()
            self._httpd = None
