"""Structured logging: one JSON object per line, with request correlation ids.

Parity: ``LoggingConfig::{development, production}``, ``Logger``, ``RequestLogger`` and the
``LogEntry`` shape (``timestamp`` ms, ``level``, ``message``, optional ``request_id``, ``module``,
``context``) of ``advanced/src/logging.rs:12-245``.  Built on Python's ``logging`` so every
module's ``logging.getLogger(...)`` output goes through the same formatter; a request id is
attached with ``request_logger(rid)`` (a ``LoggerAdapter``) or by passing
``extra={"request_id": ..., "context": {...}}``.
"""
from __future__ import annotations

import json
import logging
import sys
import time
from dataclasses import dataclass

_LEVEL_NAMES = {logging.DEBUG: "DEBUG", logging.INFO: "INFO", logging.WARNING: "WARN", logging.ERROR: "ERROR",
                logging.CRITICAL: "ERROR"}


@dataclass
class LoggingConfig:
    min_level: int = logging.INFO
    json_format: bool = True
    enable_correlation: bool = True
    log_to_stdout: bool = True
    log_file: str | None = None

    @staticmethod
    def development() -> "LoggingConfig":
        return LoggingConfig(min_level=logging.DEBUG, json_format=False)

    @staticmethod
    def production(log_file: str | None = None) -> "LoggingConfig":
        return LoggingConfig(min_level=logging.INFO, json_format=True, log_file=log_file)


class JsonFormatter(logging.Formatter):
    """``{"timestamp": ms, "level": ..., "message": ..., "request_id"?, "module"?, "context"?}``."""

    def __init__(self, correlation: bool = True):
        super().__init__()
        self.correlation = correlation

    def format(self, record: logging.LogRecord) -> str:
        entry = {"timestamp": int(record.created * 1000), "level": _LEVEL_NAMES.get(record.levelno, record.levelname),
                 "message": record.getMessage()}
        rid = getattr(record, "request_id", None)
        if self.correlation and rid:
            entry["request_id"] = str(rid)
        if record.name and record.name != "root":
            entry["module"] = record.name
        ctx = getattr(record, "context", None)
        if ctx is not None:
            entry["context"] = ctx
        if record.exc_info:
            entry.setdefault("context", {})
            if isinstance(entry["context"], dict):
                entry["context"]["exception"] = self.formatException(record.exc_info)
        return json.dumps(entry, default=str, ensure_ascii=False)


class TextFormatter(logging.Formatter):
    """``[LEVEL][request_id=...] message`` for development."""

    def format(self, record: logging.LogRecord) -> str:
        lvl = _LEVEL_NAMES.get(record.levelno, record.levelname)
        rid = getattr(record, "request_id", None)
        head = f"[{lvl}][request_id={rid}]" if rid else f"[{lvl}]"
        return f"{head} {record.getMessage()}"


_HANDLERS: list[logging.Handler] = []


def init_logger(config: LoggingConfig | None = None, name: str = "barq") -> logging.Logger:
    """Installs the formatter on the ``barq`` logger (idempotent: a second call replaces the
    handlers of the first)."""
    config = config or LoggingConfig()
    log = logging.getLogger(name)
    for h in _HANDLERS:
        log.removeHandler(h)
        h.close()
    _HANDLERS.clear()
    fmt = JsonFormatter(config.enable_correlation) if config.json_format else TextFormatter()
    if config.log_to_stdout:
        _HANDLERS.append(logging.StreamHandler(sys.stdout))
    if config.log_file:
        _HANDLERS.append(logging.FileHandler(config.log_file))
    for h in _HANDLERS:
        h.setFormatter(fmt)
        log.addHandler(h)
    log.setLevel(config.min_level)
    log.propagate = False
    return log


class _RequestAdapter(logging.LoggerAdapter):
    def process(self, msg, kwargs):
        extra = dict(kwargs.get("extra") or {})
        extra.setdefault("request_id", self.extra["request_id"])
        kwargs["extra"] = extra
        return msg, kwargs


def request_logger(request_id: str, name: str = "barq.request") -> logging.LoggerAdapter:
    """A logger whose records carry ``request_id``."""
    return _RequestAdapter(logging.getLogger(name), {"request_id": request_id})


def now_ms() -> int:
    return int(time.time() * 1000)
