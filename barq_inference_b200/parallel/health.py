"""Rank health: heartbeat watchdog over the rendezvous store, and host-side fault injection.

Parity: the reference has no rank failure detection (its health states are per-context:
``ContextManager`` Healthy/Warning/Critical, ``advanced/src/metrics.rs:220-340``).  Here every
rank of a tensor/expert/pipeline-parallel group publishes a heartbeat into the ``torch.distributed``
store; before each step a rank checks that every peer has beaten recently.  A silent peer (crashed,
exited, hung on the host, never joined) raises :class:`RankFailure` on the survivors *between*
steps, before they launch a collective that would wait for it -- no device-side wait is relied on
to notice a dead rank (the fused kernels' bounded waits are only the second line of defence).

Fault injection (``BARQ_FAULT``), always on the host so that no GPU ever faults, traps or hangs:

    BARQ_FAULT=<site>:<rank>:<step>[,...]
      kill      the rank exits (os._exit) at that step
      raise     the rank raises RuntimeError at that step
      silence   the rank stops beating (simulates a host hang) from that step on
      skip_flag the rank's fused all-reduce skips its flag write at that step (the peers' bounded
                wait then runs out and reports a timeout)
      corrupt   the request at that step gets an out-of-vocabulary token (must be rejected cleanly)
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass


class RankFailure(RuntimeError):
    """A peer rank stopped answering (no heartbeat within the timeout)."""


@dataclass(frozen=True)
class Fault:
    site: str
    rank: int
    step: int


SITES = ("kill", "raise", "silence", "skip_flag", "corrupt")


def parse_faults(spec: str | None) -> list[Fault]:
    if not spec:
        return []
    out = []
    for part in spec.split(","):
        site, rank, step = part.strip().split(":")
        if site not in SITES:
            raise ValueError(f"BARQ_FAULT: unknown site {site!r} (one of {SITES})")
        out.append(Fault(site, int(rank), int(step)))
    return out


class FaultInjector:
    def __init__(self, rank: int, spec: str | None = None):
        self.rank = rank
        self.faults = [f for f in parse_faults(spec if spec is not None else os.environ.get("BARQ_FAULT"))
                       if f.rank == rank]
        self.silenced = False

    def active(self, site: str, step: int) -> bool:
        return any(f.site == site and f.step == step for f in self.faults)

    def on_step(self, step: int) -> None:
        """Apply this rank's process-level faults due at ``step``."""
        for f in self.faults:
            if f.step != step:
                continue
            if f.site == "kill":
                os._exit(17)
            if f.site == "raise":
                raise RuntimeError(f"injected fault at step {step} on rank {self.rank}")
            if f.site == "silence":
                self.silenced = True


class Heartbeat:
    """Publishes ``hb/<rank>`` = (sequence, wall time) every ``period`` seconds from a daemon thread;
    :meth:`check` raises :class:`RankFailure` if a peer's beat is older than ``timeout``."""

    def __init__(self, store, rank: int, world: int, period: float = 0.5, timeout: float = 5.0,
                 injector: FaultInjector | None = None):
        self.store, self.rank, self.world = store, rank, world
        self.period, self.timeout = period, timeout
        self.injector = injector
        self._seq = 0
        self._stop = threading.Event()
        self._last_seen: dict[int, tuple[int, float]] = {}
        self._beat()
        self._t = threading.Thread(target=self._run, name=f"barq-heartbeat-{rank}", daemon=True)
        self._t.start()

    def _beat(self) -> None:
        if self.injector is not None and self.injector.silenced:
            return
        self._seq += 1
        self.store.set(f"hb/{self.rank}", f"{self._seq}")

    def _run(self) -> None:
        while not self._stop.wait(self.period):
            try:
                self._beat()
            except Exception:  # store gone: the process group is shutting down
                return

    def check(self, wait_join: float = 0.0) -> None:
        """Raise RankFailure naming the first peer whose beat has not advanced within the timeout.
        ``wait_join``: how long a peer that never beat at all may take to join."""
        now = time.monotonic()
        for r in range(self.world):
            if r == self.rank:
                continue
            key = f"hb/{r}"
            try:
                if not self.store.check([key]):
                    seq = None
                else:
                    seq = int(self.store.get(key))
            except Exception as e:  # noqa: BLE001 - the store itself is unreachable
                raise RankFailure(f"rank {r}: store unreachable ({e})") from e
            prev = self._last_seen.get(r)
            if seq is None:
                first = self._last_seen.setdefault(r, (-1, now))
                if now - first[1] > max(self.timeout, wait_join):
                    raise RankFailure(f"rank {r} never joined within {max(self.timeout, wait_join):.1f} s")
                continue
            if prev is None or seq != prev[0]:
                self._last_seen[r] = (seq, now)
            elif now - prev[1] > self.timeout:
                raise RankFailure(f"rank {r} silent for {now - prev[1]:.1f} s (last heartbeat #{seq})")

    def stop(self) -> None:
        self._stop.set()
