"""Continuous-batching scheduler with chunked prefill, KV admission control and preemption.

Parity: ``BatchScheduler`` (``advanced/src/continuous_batching.rs:27-180``: pending queue, admit up
to ``max_sequences``, ``fill_batch`` emitting prompts for new sequences and last tokens for running
ones, ``update_sequences`` retiring on EOS / ``max_tokens``) and its ``low_latency`` /
``high_throughput`` presets (``:213-250``).  Added: a per-step token budget with chunked prefill,
admission against free KV blocks, and preemption (recompute) of the youngest sequence when the
block pool runs dry — the reference has no memory model for its batch at all.

Each step is either a prefill step (new prompt tokens of one or more sequences) or a decode step
(one token for every running sequence); prefill has priority so TTFT stays low.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass

from .kv_cache import BlockManager
from .sequence import Sequence, SeqStatus


class Overloaded(RuntimeError):
    """Admission control refused a request (the waiting queue is full); servers answer 503."""


@dataclass
class SchedulerConfig:
    max_num_seqs: int = 64
    max_num_batched_tokens: int = 8192
    max_model_len: int = 8192
    chunked_prefill: bool = True
    # sliding-window attention: KV blocks that fall entirely out of every future query's window are
    # returned to the pool as a sequence advances (0 = no window)
    sliding_window: int = 0
    # admission control: requests beyond this many waiting are refused with Overloaded (0 = no limit)
    max_waiting: int = 0

    @staticmethod
    def low_latency() -> "SchedulerConfig":
        return SchedulerConfig(max_num_seqs=8, max_num_batched_tokens=2048)

    @staticmethod
    def high_throughput() -> "SchedulerConfig":
        return SchedulerConfig(max_num_seqs=128, max_num_batched_tokens=16384)


@dataclass
class ScheduledStep:
    kind: str  # "prefill" | "decode"
    seqs: list[Sequence]
    n_new: list[int]  # new tokens per sequence this step


class Scheduler:
    def __init__(self, cfg: SchedulerConfig, blocks: BlockManager, prefix_cache=None):
        self.cfg = cfg
        self.blocks = blocks
        self.waiting: deque[Sequence] = deque()
        self.running: list[Sequence] = []
        self.prefix_cache = prefix_cache
        self.n_preemptions = 0
        # block id written into the table entries of blocks freed by the sliding window (the
        # attention kernels never read them, but every entry must name a valid block); None
        # disables window trimming
        self.dummy_block: int | None = None
        self.n_window_freed = 0

    def add(self, seq: Sequence) -> None:
        if len(seq.prompt) == 0:
            raise ValueError("empty prompt")
        if len(seq.prompt) >= self.cfg.max_model_len:
            raise ValueError(f"prompt of {len(seq.prompt)} tokens exceeds max_model_len {self.cfg.max_model_len}")
        # a prompt whose KV pages exceed the whole pool would wait forever: refuse it up front
        usable = self.blocks.num_blocks - (1 if self.dummy_block is not None else 0)
        need = self.blocks.blocks_for(len(seq.prompt) + 1)
        if need > usable:
            raise ValueError(f"prompt of {len(seq.prompt)} tokens needs {need} KV pages; the pool has {usable}")
        if self.cfg.max_waiting and len(self.waiting) >= self.cfg.max_waiting:
            raise Overloaded(f"{len(self.waiting)} requests already waiting; retry later")
        self.waiting.append(seq)

    @property
    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def _free(self, seq: Sequence) -> None:
        if seq.block_table:
            self.blocks.release([b for i, b in enumerate(seq.block_table) if i >= seq.window_freed])
        seq.block_table = []
        seq.bt_gen += 1
        seq.n_cached = 0
        seq.window_freed = 0

    def _trim_window(self, seq: Sequence) -> None:
        """Release the blocks no future query of ``seq`` can attend to: the next query position is
        n_cached and attends to [n_cached - W + 1, n_cached], so blocks wholly below that are dead."""
        W = self.cfg.sliding_window
        if W <= 0 or self.dummy_block is None:
            return
        dead = min(max(0, seq.n_cached - W + 1) // self.blocks.block_size, len(seq.block_table))
        if dead <= seq.window_freed:
            return
        freed = seq.block_table[seq.window_freed:dead]
        self.blocks.release(freed)
        seq.block_table[seq.window_freed:dead] = [self.dummy_block] * len(freed)
        seq.bt_gen += 1
        seq.window_freed = dead
        self.n_window_freed += len(freed)

    def finish(self, seq: Sequence, reason: str) -> None:
        seq.status = SeqStatus.FINISHED
        seq.finish_reason = reason
        if self.prefix_cache is not None and seq.embeds is None and not seq.window_freed:
            self.prefix_cache.insert(seq.tokens[: seq.n_cached], seq.block_table)
        self._free(seq)
        if seq in self.running:
            self.running.remove(seq)
        elif seq in self.waiting:
            self.waiting.remove(seq)

    def abort(self, seq: Sequence) -> bool:
        """Drop a request whose client went away: a waiting one leaves the queue, a running one
        finishes with reason ``abort`` (its pages return to the pool).  False if already finished."""
        if seq.status is SeqStatus.FINISHED:
            return False
        if seq in self.waiting:
            self.waiting.remove(seq)
            seq.status = SeqStatus.FINISHED
            seq.finish_reason = "abort"
            self._free(seq)
            return True
        self.finish(seq, "abort")
        return True

    def clear_waiting(self, reason: str = "abort") -> None:
        """Drop every waiting request (engine failure or shutdown); their pages return to the pool."""
        for seq in self.waiting:
            seq.status = SeqStatus.FINISHED
            seq.finish_reason = seq.finish_reason or reason
            self._free(seq)
        self.waiting.clear()

    def _preempt_youngest(self, protect=()) -> bool:
        """Return the youngest running sequence not in ``protect`` to the front of the queue (its
        pages are freed; it recomputes on readmission)."""
        cands = [s for s in self.running if not any(s is p for p in protect)]
        if not cands:
            return False
        victim = max(cands, key=lambda s: s.arrival)
        self.running.remove(victim)
        self._free(victim)
        victim.status = SeqStatus.WAITING
        victim.n_preempted += 1
        self.n_preemptions += 1
        self.waiting.appendleft(victim)
        return True

    def schedule(self) -> ScheduledStep | None:
        cfg = self.cfg
        if cfg.sliding_window > 0:
            for s in self.running:
                self._trim_window(s)
        # 1) continue chunked prefills of running sequences first
        pre = [s for s in self.running if len(s.prompt) + len(s.output) - s.n_cached > 1]  # = n_uncached > 1
        budget = cfg.max_num_batched_tokens
        seqs, n_new = [], []
        for s in pre:
            if s.status is not SeqStatus.RUNNING:
                continue  # preempted to make room for a chunk scheduled above
            n = min(s.n_uncached, budget)
            if n <= 0:
                break
            # sequences already in this step's plan are never preempted for a later one
            if not self._reserve(s, s.n_cached + n, protect=(*seqs, s)):
                break
            seqs.append(s)
            n_new.append(n)
            budget -= n
        # 2) admit waiting sequences
        while self.waiting and budget > 0 and len(self.running) < cfg.max_num_seqs:
            s = self.waiting[0]
            if self.prefix_cache is not None and not s.block_table and s.embeds is None:
                hit_blocks, hit_tokens = self.prefix_cache.match(s.tokens[:-1])
                if hit_blocks:
                    self.blocks.retain(hit_blocks)
                    s.block_table = list(hit_blocks)
                    s.bt_gen += 1
                    s.n_cached = hit_tokens
                    s.prefix_hit = hit_tokens
            total = s.n_uncached
            n = total if total <= budget else (budget if cfg.chunked_prefill else 0)
            if n <= 0:
                break
            need = self.blocks.blocks_for(s.n_cached + n) - len(s.block_table)
            if not self.blocks.can_allocate(need):
                if self.prefix_cache is not None and self.prefix_cache.evict(need - self.blocks.n_free):
                    continue
                if s.block_table and s.prefix_hit:
                    self._free(s)
                break
            self.waiting.popleft()
            self.blocks.grow(s.block_table, s.n_cached + n)
            s.status = SeqStatus.RUNNING
            self.running.append(s)
            seqs.append(s)
            n_new.append(n)
            budget -= n
        if seqs:
            return ScheduledStep("prefill", seqs, n_new)
        # 3) decode every running sequence
        if not self.running:
            return None
        dec = []
        p0 = self.n_preemptions
        cap = self.blocks.block_size
        for s in sorted(self.running, key=lambda s: s.arrival):
            if self.n_preemptions != p0 and s.status is not SeqStatus.RUNNING:
                continue  # preempted to make room for an older sequence
            nt = len(s.prompt) + len(s.output)
            if nt <= len(s.block_table) * cap or self._reserve(s, nt):  # fast path: the page has room
                dec.append(s)
        if self.n_preemptions != p0:
            dec = [s for s in dec if s.status is SeqStatus.RUNNING]
        if not dec:
            return None
        return ScheduledStep("decode", dec, [1] * len(dec))

    def _reserve(self, s: Sequence, n_tokens: int, protect=None) -> bool:
        need = self.blocks.blocks_for(n_tokens) - len(s.block_table)
        while need > self.blocks.n_free:
            if self.prefix_cache is not None and self.prefix_cache.evict(need - self.blocks.n_free):
                continue
            if not self._preempt_youngest(protect=(s,) if protect is None else protect):
                return False
        self.blocks.grow(s.block_table, n_tokens)
        return True


_STATUS = (SeqStatus.WAITING, SeqStatus.RUNNING, SeqStatus.FINISHED)


class NativeScheduler:
    """:class:`Scheduler` whose queues, block tables, admission, window release and preemption run
    in the C++ core ``_native.Scheduler`` (``csrc/native/scheduler_native.cpp``) over the native
    block pool and radix tree.  Same decisions as the Python class (the tests replay random
    workloads through both).

    The :class:`Sequence` objects stay the engine's view: after ``schedule()`` the records of the
    sequences the core changed (status, cached length, block table and its generation, window and
    preemption counters) are copied onto them, and the cached lengths and tokens the engine wrote
    into the sequences of a plan are committed to the core before it next reads them (the next
    ``schedule()``, or ``finish()`` / ``abort()`` of that sequence).
    """

    def __init__(self, cfg: SchedulerConfig, blocks, prefix_cache=None):
        from .. import _native

        self.cfg = cfg
        self.blocks = blocks
        self.prefix_cache = prefix_cache
        self.core = _native.Scheduler(blocks.pool, prefix_cache.tree if prefix_cache is not None else None,
                                      cfg.max_num_seqs, cfg.max_num_batched_tokens, cfg.chunked_prefill,
                                      cfg.sliding_window)
        self._seqs: dict[int, Sequence] = {}
        self._ntok: dict[int, int] = {}        # tokens of each sequence that the core holds
        self._pending: dict[int, Sequence] = {}  # sequences of the last plan, not yet committed

    # ---------------------------------------------------------------- state mirrored to Python
    @property
    def dummy_block(self) -> int | None:
        b = self.core.dummy_block
        return None if b < 0 else b

    @dummy_block.setter
    def dummy_block(self, b: int | None) -> None:
        self.core.dummy_block = -1 if b is None else int(b)

    @property
    def waiting(self) -> list[Sequence]:
        """Snapshot of the waiting queue (front first); change it through the methods."""
        return [self._seqs[i] for i in self.core.waiting_ids()]

    @property
    def running(self) -> list[Sequence]:
        return [self._seqs[i] for i in self.core.running_ids()]

    @property
    def has_work(self) -> bool:
        return bool(self.core.n_waiting or self.core.n_running)

    @property
    def n_preemptions(self) -> int:
        return self.core.n_preemptions

    @property
    def n_window_freed(self) -> int:
        return self.core.n_window_freed

    def _commit(self, seqs) -> None:
        ids, cached, n_app, toks = [], [], [], []
        for s in seqs:
            known = self._ntok[s.seq_id]
            new = s.output[known - len(s.prompt):] if s.n_tokens > known else []
            ids.append(s.seq_id)
            cached.append(s.n_cached)
            n_app.append(len(new))
            toks.extend(new)
            self._ntok[s.seq_id] = known + len(new)
        if ids:
            self.core.commit(ids, cached, n_app, toks)

    def _sync_one(self, seq: Sequence) -> None:
        if self._pending.pop(seq.seq_id, None) is not None:
            self._commit((seq,))

    def _apply(self) -> None:
        for sid, st, n_cached, wf, gen, npre, phit, table in self.core.take_changes():
            s = self._seqs[sid]
            s.status = _STATUS[st]
            s.n_cached, s.window_freed, s.bt_gen = n_cached, wf, gen
            s.n_preempted, s.prefix_hit, s.block_table = npre, phit, table
            if st == 2:
                del self._seqs[sid], self._ntok[sid]
                self._pending.pop(sid, None)
                self.core.forget(sid)

    # ---------------------------------------------------------------- Scheduler interface
    def add(self, seq: Sequence) -> None:
        if len(seq.prompt) == 0:
            raise ValueError("empty prompt")
        if len(seq.prompt) >= self.cfg.max_model_len:
            raise ValueError(f"prompt of {len(seq.prompt)} tokens exceeds max_model_len {self.cfg.max_model_len}")
        usable = self.blocks.num_blocks - (1 if self.dummy_block is not None else 0)
        need = self.blocks.blocks_for(len(seq.prompt) + 1)
        if need > usable:
            raise ValueError(f"prompt of {len(seq.prompt)} tokens needs {need} KV pages; the pool has {usable}")
        if self.cfg.max_waiting and self.core.n_waiting >= self.cfg.max_waiting:
            raise Overloaded(f"{self.core.n_waiting} requests already waiting; retry later")
        self.core.add(seq.seq_id, float(seq.arrival), list(seq.tokens), seq.embeds is not None)
        self._seqs[seq.seq_id] = seq
        self._ntok[seq.seq_id] = seq.n_tokens
        self._apply()

    def finish(self, seq: Sequence, reason: str) -> None:
        seq.finish_reason = reason
        if seq.seq_id not in self._seqs:
            seq.status = SeqStatus.FINISHED
            return
        self._sync_one(seq)
        self.core.finish(seq.seq_id)
        self._apply()

    def abort(self, seq: Sequence) -> bool:
        if seq.status is SeqStatus.FINISHED or seq.seq_id not in self._seqs:
            return False
        self._sync_one(seq)
        if not self.core.abort(seq.seq_id):
            return False
        seq.finish_reason = "abort"
        self._apply()
        return True

    def clear_waiting(self, reason: str = "abort") -> None:
        for seq in self.waiting:
            seq.finish_reason = seq.finish_reason or reason
            self._sync_one(seq)
            self.core.abort(seq.seq_id)
        self._apply()

    def schedule(self) -> ScheduledStep | None:
        if self._pending:
            self._commit(self._pending.values())
            self._pending.clear()
        kind, ids, n_new = self.core.schedule()
        self._apply()
        if kind == 0:
            return None
        seqs = [self._seqs[i] for i in ids]
        self._pending = {s.seq_id: s for s in seqs}
        return ScheduledStep("prefill" if kind == 1 else "decode", seqs, list(n_new))


def new_scheduler(cfg: SchedulerConfig, blocks, prefix_cache=None):
    """The engine's scheduler: the native core when the block pool (and prefix cache) are native
    (``BARQ_NATIVE_SCHED=0`` forces the Python class)."""
    import os

    from .kv_cache import NativeBlockManager
    from .prefix_cache import NativeRadixPrefixCache

    native = (os.environ.get("BARQ_NATIVE_SCHED", "1") != "0" and isinstance(blocks, NativeBlockManager)
              and (prefix_cache is None or isinstance(prefix_cache, NativeRadixPrefixCache)))
    if native:
        from .. import _native

        native = hasattr(_native, "Scheduler")
    return (NativeScheduler if native else Scheduler)(cfg, blocks, prefix_cache)
