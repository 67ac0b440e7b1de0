"""Paged KV-cache block manager.

Parity: the reference's ``PagedAttention`` page pool (``advanced/src/paged_attention.rs:27-212``:
alloc/free per sequence, defrag), ``AdvancedKVCache`` (``models/src/kv_cache.rs:169-505``) and the
contiguous per-context ``KVCache`` (``models/src/context.rs:245-339``).  Blocks of 16 tokens with
reference counts, so prefix blocks can be shared between sequences (radix prefix cache) and freed
when the last user releases them.  There is no defragmentation: block tables make physical
placement irrelevant to the kernels, so fragmentation never blocks an allocation.
"""
from __future__ import annotations

from dataclasses import dataclass, field


class OutOfBlocks(RuntimeError):
    pass


@dataclass
class BlockManager:
    num_blocks: int
    block_size: int = 16
    free: list[int] = field(default_factory=list)
    ref: list[int] = field(default_factory=list)

    def __post_init__(self):
        self.free = list(range(self.num_blocks - 1, -1, -1))
        self.ref = [0] * self.num_blocks

    @property
    def n_free(self) -> int:
        return len(self.free)

    @property
    def n_used(self) -> int:
        return self.num_blocks - len(self.free)

    def blocks_for(self, n_tokens: int) -> int:
        return (n_tokens + self.block_size - 1) // self.block_size

    def can_allocate(self, n: int) -> bool:
        return n <= len(self.free)

    def allocate(self, n: int) -> list[int]:
        if n > len(self.free):
            raise OutOfBlocks(f"need {n} blocks, {len(self.free)} free")
        out = [self.free.pop() for _ in range(n)]
        for b in out:
            self.ref[b] = 1
        return out

    def retain(self, blocks: list[int]) -> None:
        for b in blocks:
            if self.ref[b] <= 0:
                raise ValueError(f"retain of free block {b}")
            self.ref[b] += 1

    def release(self, blocks: list[int]) -> None:
        for b in blocks:
            if self.ref[b] <= 0:
                raise ValueError(f"double free of block {b}")
            self.ref[b] -= 1
            if self.ref[b] == 0:
                self.free.append(b)

    def grow(self, table: list[int], n_tokens: int) -> list[int]:
        """Extend ``table`` so it covers ``n_tokens`` tokens; returns the new blocks."""
        need = self.blocks_for(n_tokens) - len(table)
        if need <= 0:
            return []
        new = self.allocate(need)
        table.extend(new)
        return new

    def stats(self) -> dict:
        return {"num_blocks": self.num_blocks, "used": self.n_used, "free": self.n_free,
                "block_size": self.block_size, "usage": self.n_used / max(1, self.num_blocks)}


def _native_kv():
    import os

    if os.environ.get("BARQ_NATIVE_KV", "1") == "0":
        return None
    try:
        import torch  # noqa: F401  (the extension links against torch's libraries: load them first)

        from .. import _native
    except ImportError:
        return None
    return _native if hasattr(_native, "BlockPool") else None


class NativeBlockManager:
    """:class:`BlockManager` backed by the C++ ``_native.BlockPool`` (same contract, same block ids)."""

    def __init__(self, num_blocks: int, block_size: int = 16):
        self.pool = _native_kv().BlockPool(num_blocks, block_size)
        self.num_blocks, self.block_size = num_blocks, block_size

    @property
    def n_free(self) -> int:
        return self.pool.n_free

    @property
    def n_used(self) -> int:
        return self.pool.n_used

    @property
    def ref(self) -> list[int]:
        return self.pool.refs()

    @property
    def free(self) -> list[int]:
        return self.pool.free_list()

    def blocks_for(self, n_tokens: int) -> int:
        return self.pool.blocks_for(n_tokens)

    def can_allocate(self, n: int) -> bool:
        return self.pool.can_allocate(n)

    def allocate(self, n: int) -> list[int]:
        try:
            return self.pool.allocate(n)
        except IndexError as e:  # std::out_of_range
            raise OutOfBlocks(str(e)) from None

    def retain(self, blocks: list[int]) -> None:
        self.pool.retain(blocks)

    def release(self, blocks: list[int]) -> None:
        self.pool.release(blocks)

    def grow(self, table: list[int], n_tokens: int) -> list[int]:
        need = self.pool.blocks_for(n_tokens) - len(table)
        if need <= 0:
            return []
        new = self.allocate(need)
        table.extend(new)
        return new

    def stats(self) -> dict:
        used = self.pool.n_used
        return {"num_blocks": self.num_blocks, "used": used, "free": self.pool.n_free,
                "block_size": self.block_size, "usage": used / max(1, self.num_blocks)}


def new_block_manager(num_blocks: int, block_size: int = 16):
    """The engine's block manager: the native pool when ``_native`` is built (``BARQ_NATIVE_KV=0``
    forces the Python one)."""
    return NativeBlockManager(num_blocks, block_size) if _native_kv() is not None else \
        BlockManager(num_blocks, block_size)
