"""Build and locate the native front-end tools of the UDS server:

* ``barq-uds`` (``csrc/client/barq_uds.cpp``): command-line client;
* ``barq-http`` (``csrc/client/barq_http.cpp``): OpenAI-compatible HTTP front end that forwards
  every generation to the UDS server.

The binaries are compiled in-tree next to this package (``barq_inference_b200/bin/``) so that they
travel with the checkout; the package build entry point and the tests call ``build_client()`` /
``build_http()``, which rebuild a binary when it is missing or older than its sources.
"""
from __future__ import annotations

import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCE = os.path.join(os.path.dirname(PKG), "csrc", "client", "barq_uds.cpp")
BINARY = os.path.join(PKG, "bin", "barq-uds")
HTTP_SOURCES = [os.path.join(os.path.dirname(PKG), "csrc", "client", f) for f in ("barq_http.cpp", "json_lite.h")]
HTTP_BINARY = os.path.join(PKG, "bin", "barq-http")


def _compile(cmd: list[str], out: str) -> None:
    """Compile to a private file and rename it into place: concurrent builders (parallel test
    workers) never run or overwrite a half-written binary."""
    tmp = f"{out}.{os.getpid()}.tmp"
    try:
        subprocess.run([*cmd, "-o", tmp], check=True)
        os.replace(tmp, out)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)


def client_path() -> str:
    return BINARY


def build_client(force: bool = False) -> str:
    """Compile the client with the host C++ compiler if it is missing or stale; returns its path."""
    fresh = (os.path.exists(BINARY) and os.path.exists(SOURCE)
             and os.path.getmtime(BINARY) >= os.path.getmtime(SOURCE))
    if fresh and not force:
        return BINARY
    cxx = os.environ.get("CXX") or shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("no C++ compiler found to build barq-uds")
    os.makedirs(os.path.dirname(BINARY), exist_ok=True)
    _compile([cxx, "-O2", "-std=c++17", "-Wall", "-Wextra", "-Werror", SOURCE], BINARY)
    return BINARY


def http_path() -> str:
    return HTTP_BINARY


def build_http(force: bool = False) -> str:
    """Compile ``barq-http`` if it is missing or older than its sources; returns its path."""
    fresh = os.path.exists(HTTP_BINARY) and all(
        os.path.exists(src) and os.path.getmtime(HTTP_BINARY) >= os.path.getmtime(src) for src in HTTP_SOURCES)
    if fresh and not force:
        return HTTP_BINARY
    cxx = os.environ.get("CXX") or shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        raise RuntimeError("no C++ compiler found to build barq-http")
    os.makedirs(os.path.dirname(HTTP_BINARY), exist_ok=True)
    _compile([cxx, "-O2", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-pthread", HTTP_SOURCES[0]], HTTP_BINARY)
    return HTTP_BINARY
