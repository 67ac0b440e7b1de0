"""Loopback model of the fused push all-reduce protocol, for testing its host-visible logic on CPU.

The decode row-parallel GEMV (``csrc/kernels/gemv_stream.cu``, ``EPI_AR_PUSH``) exchanges results
with this protocol; this module runs the same steps with one thread per rank over shared numpy
arrays, so ordering, epochs, timeouts and buffer reuse can be exercised with random per-rank
delays and no GPU:

* rank r owns receive buffers ``recv[r][j]`` of 64-bit words, one slot per (source rank, batch
  row, output row); a word is ``epoch << 32 | float32 bits`` (the value and its epoch travel in one
  store, so a reader that sees the epoch sees the value: no fence, no flag);
* a call on buffer j uses epoch ``epoch[r][j] + 1``; the rank walks its 128-row tiles in
  increasing order, for each tile stores its words into every peer's ``recv[q][j]`` slot r, then
  waits (bounded) for every peer's words of that tile carrying exactly this epoch, and adds the
  tile's sum — in rank order, so every rank computes bit-identical sums — into its residual x;
* a wait that runs out records ``0x300 | peer`` in the rank's error word and leaves that row's x
  unchanged; the epoch still advances at the end of the call, so ranks stay aligned;
* reuse rule: between two calls on the same buffer every rank must pass some other collective.
  Without it a fast rank can overwrite a slot with the next epoch before a slow peer has read the
  previous one; the slow peer then never sees its epoch and times out (an error, never a wrong sum).
"""
from __future__ import annotations

import random
import threading
import time

import numpy as np

TILE = 128


def pack(epoch: int, v: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(v, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return (np.uint64(epoch) << np.uint64(32)) | bits


def unpack(words: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    ep = (words >> np.uint64(32)).astype(np.uint32)
    val = (words & np.uint64(0xFFFFFFFF)).astype(np.uint32).view(np.float32)
    return ep, val


class LoopbackFabric:
    """Receive buffers, epochs and error words of ``world`` ranks sharing one address space."""

    def __init__(self, world: int, n_bufs: int, B: int, N: int):
        if N % TILE:
            raise ValueError(f"N must be a multiple of {TILE}")
        self.world, self.B, self.N = world, B, N
        self.recv = [[np.zeros((world, B, N), np.uint64) for _ in range(n_bufs)] for _ in range(world)]
        self.epoch = [[0] * n_bufs for _ in range(world)]
        self.err = [0] * world
        self._lock = threading.Lock()  # stands in for 64-bit store atomicity of a tile's words

    def push_allreduce(self, rank: int, j: int, partial: np.ndarray, x: np.ndarray, wait_s: float = 2.0,
                       skip_signal: bool = False, jitter_s: float = 0.0, rng: random.Random | None = None,
                       pause_after_write_s: float = 0.0) -> None:
        """x[b, :] += sum over ranks of partial_r[b, :] (the rank's own ``partial`` [B, N] fp32)."""
        W, B, N = self.world, self.B, self.N
        ep = self.epoch[rank][j] + 1
        own = partial.astype(np.float32)
        for t in range(N // TILE):
            sl = slice(t * TILE, (t + 1) * TILE)
            if jitter_s and rng is not None:
                time.sleep(rng.random() * jitter_s)
            if not skip_signal:
                words = pack(ep, own[:, sl])
                with self._lock:
                    for q in range(W):
                        if q != rank:
                            self.recv[q][j][rank, :, sl] = words
            if pause_after_write_s:
                time.sleep(pause_after_write_s)
            got = {}
            ok = True
            for q in range(W):
                if q == rank:
                    continue
                deadline = time.monotonic() + wait_s
                while True:
                    with self._lock:
                        e, v = unpack(self.recv[rank][j][q, :, sl].copy())
                    if np.all(e == ep):
                        got[q] = v
                        break
                    # like the kernel: give up at the deadline, or at once when an earlier wait
                    # of this rank already failed (its error word is set)
                    if time.monotonic() > deadline or (self.err[rank] & 0xF00) == 0x300:
                        if not self.err[rank]:
                            self.err[rank] = 0x300 | q
                        ok = False
                        break
                    time.sleep(0.0002)
                if not ok:
                    break
            if ok:
                s = np.zeros((B, TILE), np.float32)
                for q in range(W):  # rank order on every rank
                    s += own[:, sl] if q == rank else got[q]
                x[:, sl] += s
        self.epoch[rank][j] = ep


def run_ranks(fabric: LoopbackFabric, fn, seed: int = 0) -> list:
    """Runs ``fn(rank, rng)`` on one thread per rank; returns the per-rank results (re-raising the
    first exception)."""
    out: list = [None] * fabric.world
    errs: list = []

    def body(r):
        try:
            out[r] = fn(r, random.Random(seed * 1000 + r))
        except BaseException as e:  # noqa: BLE001 - reported to the caller
            errs.append(e)

    th = [threading.Thread(target=body, args=(r,)) for r in range(fabric.world)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    if errs:
        raise errs[0]
    return out
