"""Loopback model of the sequence-parallel reduce-scatter / all-gather protocol, for CPU tests.

The fused tensor-parallel path (``csrc/kernels/tp_fused.cu`` and the ``EPI_RS_PUSH`` / ``SpWait``
modes of ``csrc/kernels/gemm_tc.cu``) reuses its receive slots and gather buffers from layer to
layer without any barrier, relying on data dependencies alone.  This module runs the same protocol
with one thread per rank over shared numpy arrays, with random per-rank delays and a random tile
order inside every "kernel", so that the reuse argument can be checked on CPU:

* a row-parallel GEMM of rank s at site j (epoch ``e = epoch[s][j] + 1``) walks its output tiles
  in any order; for each it writes the tile's rows of its partial into ``slots[o][s]`` of the
  owner o of those rows (tagged with e) and then sets ``rs_flag[o][j][s][tile] = e``;
* the owner's reduce (same epoch rule) waits for the flags of the tiles covering each of its rows
  from every source rank, checks that every slot row it reads carries tag e (a stale or
  overwritten slot would show here), adds the partials in rank order into its residual rows,
  normalizes them and pushes the row into every rank's gather buffer (tagged e) followed by the
  row flag, then advances ``epoch[o][j]``;
* the next column-parallel GEMM of every rank waits per token tile for the row flags carrying the
  epoch of its local counter and checks the tags of the rows it reads.

A tag mismatch is a protocol violation (``ProtocolError``); a wait that runs out is a timeout
(``TimeoutError``).  Neither should happen for any interleaving: a rank writes a peer's slots or
gather rows for call c+1 only after a chain of waits that starts at that peer's reads of call c.
"""
from __future__ import annotations

import random
import threading
import time

import numpy as np


class ProtocolError(RuntimeError):
    pass


class SpFabric:
    def __init__(self, world: int, T: int, H: int, bn: int = 4, tile_n: int = 128, seed: int = 0):
        self.W, self.T, self.H, self.bn, self.tile_n = world, T, H, bn, tile_n
        self.chunk = -(-T // world)
        self.t_tiles, self.n_tiles = -(-T // bn), -(-H // tile_n)
        W, c = world, self.chunk
        self.slots = np.zeros((W, W, c, H), np.float32)            # [owner][src][row][col]
        self.slot_tag = np.zeros((W, W, c, self.n_tiles), np.int64)  # epoch of each (row, n tile) piece
        self.rs_flag = np.zeros((W, 2, W, self.n_tiles * self.t_tiles), np.int64)
        self.ag = np.zeros((W, 2, T, H), np.float32)                # [rank][site][row][col]
        self.ag_tag = np.zeros((W, 2, T), np.int64)
        self.ag_flag = np.zeros((W, 2, T), np.int64)
        self.epoch = np.zeros((W, 2), np.int64)
        self.rng = [random.Random(seed * 1000 + r) for r in range(W)]

    # ---------------------------------------------------------------- helpers
    def _nap(self, r: int, scale: float) -> None:
        if scale > 0:
            time.sleep(self.rng[r].random() * scale)

    @staticmethod
    def _wait(pred, limit: float, what: str) -> None:
        t0 = time.monotonic()
        while not pred():
            if time.monotonic() - t0 > limit:
                raise TimeoutError(what)
            time.sleep(0)

    def rows_of(self, r: int) -> range:
        a = min(self.T, r * self.chunk)
        return range(a, min(self.T, a + self.chunk))

    # ---------------------------------------------------------------- the three kernels
    def gemm_rs(self, s: int, j: int, partial: np.ndarray, jitter: float = 0.0) -> None:
        """Row-parallel GEMM of rank s: push every output tile of ``partial`` [T, H] to its owners."""
        e = self.epoch[s][j] + 1
        tiles = [(tt, nt) for tt in range(self.t_tiles) for nt in range(self.n_tiles)]
        self.rng[s].shuffle(tiles)
        for tt, nt in tiles:
            self._nap(s, jitter)
            r0, r1 = tt * self.bn, min(self.T, (tt + 1) * self.bn)
            c0, c1 = nt * self.tile_n, min(self.H, (nt + 1) * self.tile_n)
            owners = set()
            for t in range(r0, r1):
                o = t // self.chunk
                self.slots[o, s, t - o * self.chunk, c0:c1] = partial[t, c0:c1]
                self.slot_tag[o, s, t - o * self.chunk, nt] = e
                owners.add(o)
            for o in owners:  # flag after the data (the kernel fences at system scope here)
                self.rs_flag[o, j, s, nt + self.n_tiles * tt] = e

    def reduce_norm_ag(self, o: int, j: int, x: np.ndarray, norm_w: np.ndarray, reduce: bool = True,
                       jitter: float = 0.0, wait_s: float = 5.0) -> None:
        """Owner o: x (its rows, [rows, H]) += partials in rank order; RMSNorm; push to every rank."""
        e = self.epoch[o][j] + 1
        rows = list(self.rows_of(o))
        order = list(range(len(rows)))
        self.rng[o].shuffle(order)
        for lr in order:
            self._nap(o, jitter)
            t = rows[lr]
            if reduce:
                tt = t // self.bn
                for s in range(self.W):
                    for nt in range(self.n_tiles):
                        f = (o, j, s, nt + self.n_tiles * tt)
                        self._wait(lambda f=f: self.rs_flag[f] >= e, wait_s, f"rs flag {f} epoch {e}")
                for s in range(self.W):  # rank order: the same sum on every rank
                    if (self.slot_tag[o, s, lr] != e).any():
                        raise ProtocolError(f"owner {o} row {t}: slot of rank {s} tagged "
                                            f"{self.slot_tag[o, s, lr].tolist()}, expected {e}")
                    x[lr] += self.slots[o, s, lr]
            v = x[lr]
            y = v / np.sqrt((v * v).mean() + 1e-5) * norm_w
            for q in range(self.W):
                self.ag[q, j, t] = y
                self.ag_tag[q, j, t] = e
            for q in range(self.W):
                self.ag_flag[q, j, t] = e
        self.epoch[o][j] = e

    def gemm_ag(self, r: int, j: int, jitter: float = 0.0, wait_s: float = 5.0) -> np.ndarray:
        """Column-parallel GEMM of rank r: read the gathered rows tile by tile once they arrived."""
        e = self.epoch[r][j]
        out = np.empty((self.T, self.H), np.float32)
        tiles = list(range(self.t_tiles))
        self.rng[r].shuffle(tiles)
        for tt in tiles:
            self._nap(r, jitter)
            r0, r1 = tt * self.bn, min(self.T, (tt + 1) * self.bn)
            for t in range(r0, r1):
                self._wait(lambda t=t: self.ag_flag[r, j, t] >= e, wait_s, f"ag flag rank {r} row {t}")
            if (self.ag_tag[r, j, r0:r1] != e).any():
                raise ProtocolError(f"rank {r} rows {r0}..{r1}: gathered rows tagged "
                                    f"{self.ag_tag[r, j, r0:r1].tolist()}, expected {e}")
            out[r0:r1] = self.ag[r, j, r0:r1]
        return out


def run_layers(world: int, T: int, H: int, layers: int, seed: int = 0, jitter: float = 2e-4,
               bn: int = 4) -> tuple[list[np.ndarray], np.ndarray]:
    """Run ``layers`` Megatron layers (two sites each) of the protocol on ``world`` threads.

    Every rank's row-parallel partials are a fixed function of the gathered input it read, so the
    threaded run must reproduce the sequential reference (to float32 rounding).  Returns the
    per-rank residual rows after the last layer (in rank order) and the reference residual."""
    fab = SpFabric(world, T, H, bn=bn, seed=seed)
    g = np.random.default_rng(seed)
    x0 = g.standard_normal((T, H)).astype(np.float32)
    norms = [(1 + 0.1 * g.standard_normal(H)).astype(np.float32) for _ in range(2 * layers + 1)]
    mats = [[(0.05 * g.standard_normal((H, H))).astype(np.float32) for _ in range(world)]
            for _ in range(2 * layers)]

    def rms(v, w):
        return v / np.sqrt((v * v).mean(-1, keepdims=True) + 1e-5) * w

    # sequential reference
    ref = x0.copy()
    h = rms(ref, norms[0])
    for k in range(2 * layers):
        for s in range(world):  # rank order, added one partial at a time like the owner kernel
            ref = ref + h @ mats[k][s]
        h = rms(ref, norms[k + 1])

    xs = [x0[list(fab.rows_of(r))].copy() for r in range(world)]
    errors: list[BaseException] = []

    def rank_main(r: int) -> None:
        try:
            fab.reduce_norm_ag(r, 1, xs[r], norms[0], reduce=False, jitter=jitter)
            site_in = 1
            for k in range(2 * layers):
                hin = fab.gemm_ag(r, site_in, jitter=jitter)           # column-parallel input
                fab.gemm_rs(r, k % 2, hin @ mats[k][r], jitter=jitter)  # row-parallel output
                fab.reduce_norm_ag(r, k % 2, xs[r], norms[k + 1], jitter=jitter)
                site_in = k % 2
        except BaseException as exc:  # noqa: BLE001 - reported to the caller
            errors.append(exc)

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    if errors:
        raise errors[0]
    return [xs[r] for r in range(world)], ref
