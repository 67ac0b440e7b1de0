"""Build and locate ``barq-uds``, the native client of the UDS server (``csrc/client/barq_uds.cpp``).

The binary is compiled in-tree next to this package (``barq_inference_b200/bin/barq-uds``) so that
it travels with the checkout; ``build_client()`` is called by the package build entry point and by
the tests when the binary is missing or older than its source.
"""
from __future__ import annotations

import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SOURCE = os.path.join(os.path.dirname(PKG), "csrc", "client", "barq_uds.cpp")
BINARY = os.path.join(PKG, "bin", "barq-uds")


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
    subprocess.run([cxx, "-O2", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-o", BINARY, SOURCE], check=True)
    return BINARY
