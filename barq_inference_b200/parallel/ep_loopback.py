"""Loopback model of the expert-parallel all-to-all protocol (``csrc/kernels/moe.cu`` ``ep_*``).

One thread per rank over shared numpy arrays, random per-rank delays and random row order inside
every "kernel", MoE layers run back to back with no barrier:

* counts: rank s writes its per-expert row counts into row s of every rank's count matrix, then
  sets ``cnt_flag[q][s] = e`` (``e`` = the rank's EP call counter + 1);
* dispatch: rank s waits for every rank's count flag, derives the receive row of each of its
  (token, slot) pairs (expert owner's receive rows in expert-major, then source-rank order -- the
  kernel's ``ep_base``), copies the token row there (tagged e), flags ``disp_flag[o][s] = e`` at
  every owner, then waits for every rank's dispatch flag into its own rows;
* the experts run on the received rows (here: expert x scales a row by x + 1) -- rows tagged e
  only, anything else is a ``ProtocolError``;
* signal + combine: rank s marks its outputs ready at every rank, waits for every rank's mark, and
  gathers gate_weight * output of each of its slots from the owners, in slot order.

The threaded result must match a sequential reference, and the epoch tags show any row that a
fast rank overwrote before its owner used it.
"""
from __future__ import annotations

import random
import threading
import time

import numpy as np


class ProtocolError(RuntimeError):
    pass


def recv_row_base(cm: np.ndarray, E_local: int, e: int, src: int) -> int:
    """Receive row of the first row that rank ``src`` sends to expert e (on e's owner): the rows of
    the owner's lower experts from every rank, then expert e's rows of ranks below ``src``."""
    e0 = (e // E_local) * E_local
    return int(cm[:, e0:e].sum() + cm[:src, e].sum())


class EpFabric:
    def __init__(self, world: int, E: int, k: int, rows: int, H: int, seed: int = 0):
        self.W, self.E, self.k, self.rows, self.H = world, E, k, rows, H
        self.El = E // world
        cap = world * rows * k
        self.cm = np.zeros((world, world, E), np.int64)          # [rank][src][expert]
        self.cnt_flag = np.zeros((world, world), np.int64)
        self.recv = np.zeros((world, cap, H), np.float32)
        self.recv_tag = np.zeros((world, cap), np.int64)
        self.disp_flag = np.zeros((world, world), np.int64)
        self.ys = np.zeros((world, cap, H), np.float32)
        self.ys_tag = np.zeros((world, cap), np.int64)
        self.ys_flag = np.zeros((world, world), np.int64)
        self.epoch = np.zeros(world, np.int64)
        self.rng = [random.Random(seed * 7919 + r) for r in range(world)]

    def _nap(self, r, scale):
        if scale > 0:
            time.sleep(self.rng[r].random() * scale)

    @staticmethod
    def _wait(pred, limit, what):
        t0 = time.monotonic()
        while not pred():
            if time.monotonic() - t0 > limit:
                raise TimeoutError(what)
            time.sleep(0)

    def layer(self, s: int, x: np.ndarray, ids: np.ndarray, w: np.ndarray, jitter: float = 0.0,
              wait_s: float = 5.0) -> np.ndarray:
        """One MoE layer of rank s: returns sum_j w[t, j] * expert_{ids[t, j]}(x[t]) for its rows."""
        W, E, k, El = self.W, self.E, self.k, self.El
        e = self.epoch[s] + 1
        counts = np.bincount(ids[w > 0], minlength=E)
        for q in range(W):  # counts -> every rank, then the flag
            self.cm[q, s] = counts
        for q in range(W):
            self.cnt_flag[q, s] = e
        for q in range(W):
            self._wait(lambda q=q: self.cnt_flag[s, q] >= e, wait_s, f"count flag {s}<-{q}")
        cm = self.cm[s].copy()
        cursor = np.zeros(E, np.int64)
        pos = np.full((len(x), k), -1, np.int64)
        order = [(t, j) for t in range(len(x)) for j in range(k)]
        self.rng[s].shuffle(order)
        for t, j in order:  # dispatch
            self._nap(s, jitter)
            if w[t, j] <= 0:
                continue
            ex = int(ids[t, j])
            o = ex // El
            p = recv_row_base(cm, El, ex, s) + cursor[ex]
            cursor[ex] += 1
            self.recv[o, p] = x[t]
            self.recv_tag[o, p] = e
            pos[t, j] = p
        for o in range(W):
            self.disp_flag[o, s] = e
        for q in range(W):
            self._wait(lambda q=q: self.disp_flag[s, q] >= e, wait_s, f"dispatch flag {s}<-{q}")
        # the experts of rank s on its received rows
        e0 = s * El
        n_recv = int(cm[:, e0:e0 + El].sum())
        off = [recv_row_base(cm, El, e0 + i, 0) for i in range(El)] + [n_recv]  # the kernel's recv_off
        for p in range(n_recv):
            if self.recv_tag[s, p] != e:
                raise ProtocolError(f"rank {s} receive row {p} tagged {self.recv_tag[s, p]}, expected {e}")
            ex = e0 + max(i for i in range(El) if off[i] <= p)
            self.ys[s, p] = self.recv[s, p] * (ex + 1)
            self.ys_tag[s, p] = e
        for q in range(W):  # outputs ready
            self.ys_flag[q, s] = e
        for q in range(W):
            self._wait(lambda q=q: self.ys_flag[s, q] >= e, wait_s, f"output flag {s}<-{q}")
        out = np.zeros_like(x)
        for t in range(len(x)):  # combine in slot order
            for j in range(k):
                if pos[t, j] < 0:
                    continue
                o = int(ids[t, j]) // El
                if self.ys_tag[o, pos[t, j]] != e:
                    raise ProtocolError(f"rank {s} token {t} slot {j}: output row tagged "
                                        f"{self.ys_tag[o, pos[t, j]]}, expected {e}")
                out[t] += w[t, j] * self.ys[o, pos[t, j]]
        self.epoch[s] = e
        return out


def run_layers(world: int, E: int, k: int, rows: int, H: int, layers: int, seed: int = 0,
               jitter: float = 2e-4) -> tuple[list[np.ndarray], list[np.ndarray]]:
    """``layers`` MoE layers on ``world`` threads; returns (threaded outputs, sequential reference)
    per rank of the last layer's residual rows."""
    fab = EpFabric(world, E, k, rows, H, seed=seed)
    g = np.random.default_rng(seed)
    xs = [g.standard_normal((rows, H)).astype(np.float32) for _ in range(world)]
    routes = [[(g.integers(0, E, (rows, k)), np.where(g.random((rows, k)) < 0.15, 0.0, g.random((rows, k))))
               for _ in range(world)] for _ in range(layers)]
    ref = [x.copy() for x in xs]
    for li in range(layers):
        for s in range(world):
            ids, w = routes[li][s]
            add = np.zeros_like(ref[s])
            for t in range(rows):
                for j in range(k):
                    if w[t, j] > 0:
                        add[t] += w[t, j] * (ref[s][t] * (ids[t, j] + 1))
            ref[s] = ref[s] + add
    got = [x.copy() for x in xs]
    errors: list[BaseException] = []

    def rank_main(s):
        try:
            for li in range(layers):
                ids, w = routes[li][s]
                got[s] = got[s] + fab.layer(s, got[s], ids, w, jitter=jitter)
        except BaseException as exc:  # noqa: BLE001 - reported to the caller
            errors.append(exc)

    ths = [threading.Thread(target=rank_main, args=(s,)) for s in range(world)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    if errors:
        raise errors[0]
    return got, ref
