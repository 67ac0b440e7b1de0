"""Serving a model that spans several ranks (tensor / pipeline parallel): rank 0 runs the server and
every other rank replays its scheduler inputs in lockstep.

Every rank of a tensor- or pipeline-parallel engine runs its own (replicated) scheduler and must
take exactly the same steps over exactly the same requests, because each step's forward contains
collectives.  ``LockstepLeader`` wraps rank 0's engine: the requests added since the previous step
are published through the process group's key-value store under a step number before the step
runs; ``follower_loop`` on the other ranks reads step k's commands, applies them and runs step k.
While the server is idle nobody steps and followers wait on the store (no collective is pending,
so no process-group timeout can fire).  Sampling needs no exchange: logits are gathered on every
rank and seeds derive from the same request ids, so every rank samples the same tokens.

Commands: ("add", prompt, params, request_id, embeds, leader's sequence id) | ("reset",) after a
failed step (followers drop their requests, as the leader's server does) | ("stop",).
"""
from __future__ import annotations

import datetime
import pickle

_PREFIX = "barq/lockstep/"


def _key(k: int) -> str:
    return f"{_PREFIX}{k}"


class LockstepLeader:
    """Rank 0's engine as the server sees it; forwards everything else to the wrapped engine."""

    def __init__(self, engine, store, keep: int = 64):
        self.engine = engine
        self.store = store
        self.k = 0
        self.keep = keep  # old command keys are deleted this many steps later
        self.pending: list = []

    def __getattr__(self, name):
        return getattr(self.engine, name)

    def add_request(self, prompt, params=None, request_id: str = "", on_token=None, embeds=None):
        seq = self.engine.add_request(prompt, params, request_id, on_token=on_token, embeds=embeds)  # validates
        e = None if embeds is None else (int(embeds[0]), embeds[1].detach().float().cpu())
        self.pending.append(("add", list(prompt), seq.params, request_id, e, seq.seq_id))
        return seq

    def _publish(self, cmds: list) -> None:
        self.store.set(_key(self.k), pickle.dumps(cmds))
        if self.k >= self.keep:
            try:
                self.store.delete_key(_key(self.k - self.keep))
            except Exception:  # noqa: BLE001 - a store without delete keeps the key
                pass
        self.k += 1

    def step(self):
        cmds, self.pending = self.pending, []
        self._publish(cmds)
        try:
            return self.engine.step()
        except Exception:
            self.pending.append(("reset",))
            raise

    def has_work(self) -> bool:
        return self.engine.has_work() or bool(self.pending)

    def stop(self) -> None:
        self._publish(self.pending + [("stop",)])
        self.pending = []


def _reset(engine) -> None:
    sched = getattr(engine, "sched", None)
    if sched is None:
        return
    for s in list(sched.running):
        sched.finish(s, "error")
    sched.clear_waiting("error")


def follower_loop(engine, store, wait_s: float = 7 * 24 * 3600.0, collect: list | None = None) -> int:
    """Replays rank 0's steps on this rank until it publishes ``stop``; returns the steps taken.
    ``collect`` (a list) receives this rank's sequences in the order they were added."""
    store.set_timeout(datetime.timedelta(seconds=wait_s))
    k = 0
    while True:
        cmds = pickle.loads(store.get(_key(k)))
        k += 1
        for c in cmds:
            if c[0] == "stop":
                return k - 1
            if c[0] == "reset":
                _reset(engine)
            elif c[0] == "add":
                _, prompt, params, rid, embeds, seq_id = c
                # the leader's sequence id: sampling seeds derive from it, so every rank draws alike
                seq = engine.add_request(prompt, params, rid, embeds=embeds)
                seq.seq_id = seq_id
                if collect is not None:
                    collect.append(seq)
        try:
            engine.step()
        except Exception:  # noqa: BLE001 - the leader fails too and publishes a reset
            pass
