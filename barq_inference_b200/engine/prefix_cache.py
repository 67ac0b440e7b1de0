"""Radix prefix cache over paged KV blocks.

Parity: ``PromptCache`` (``advanced/src/prompt_cache.rs:16-258``: radix tree of token edges -> KV page
ids, longest-prefix match, incremental insert, LRU eviction by page budget).  Here nodes hold whole
16-token blocks of the paged KV cache; a finished sequence donates its full blocks (the cache keeps
a reference), a new request reuses the longest cached block-aligned prefix (its blocks are retained
by the sequence), and eviction frees least-recently-used leaves whose blocks no running sequence uses.
"""
from __future__ import annotations

import itertools
from dataclasses import dataclass, field

from .kv_cache import BlockManager

_clock = itertools.count()


@dataclass
class _Node:
    key: tuple[int, ...] = ()
    block: int = -1
    parent: "_Node | None" = None
    children: dict = field(default_factory=dict)
    last_used: int = 0


class RadixPrefixCache:
    def __init__(self, blocks: BlockManager):
        self.bm = blocks
        self.bs = blocks.block_size
        self.root = _Node()
        self.n_blocks = 0
        self.hits = 0
        self.queries = 0

    def match(self, tokens: list[int]) -> tuple[list[int], int]:
        """Longest cached block-aligned prefix: (block ids, number of tokens)."""
        self.queries += 1
        node, out = self.root, []
        for i in range(0, len(tokens) - self.bs + 1, self.bs):
            key = tuple(tokens[i:i + self.bs])
            child = node.children.get(key)
            if child is None:
                break
            child.last_used = next(_clock)
            out.append(child.block)
            node = child
        if out:
            self.hits += 1
        return out, len(out) * self.bs

    def insert(self, tokens: list[int], block_table: list[int]) -> None:
        """Donate the full blocks of a finished sequence (the cache takes its own reference)."""
        node = self.root
        n_full = min(len(tokens) // self.bs, len(block_table))
        for j in range(n_full):
            key = tuple(tokens[j * self.bs:(j + 1) * self.bs])
            child = node.children.get(key)
            if child is None:
                child = _Node(key, block_table[j], node)
                node.children[key] = child
                self.bm.retain([child.block])
                self.n_blocks += 1
            child.last_used = next(_clock)
            node = child

    def evict(self, n: int) -> int:
        """Free up to n blocks from least-recently-used leaves no one else references."""
        freed = 0
        while freed < n:
            leaves = []
            stack = [self.root]
            while stack:
                nd = stack.pop()
                if not nd.children and nd is not self.root:
                    leaves.append(nd)
                stack.extend(nd.children.values())
            cands = [lf for lf in leaves if self.bm.ref[lf.block] == 1]
            if not cands:
                break
            victim = min(cands, key=lambda x: x.last_used)
            del victim.parent.children[victim.key]
            self.bm.release([victim.block])
            self.n_blocks -= 1
            freed += 1
        return freed

    def stats(self) -> dict:
        return {"cached_blocks": self.n_blocks, "queries": self.queries, "hits": self.hits,
                "hit_rate": self.hits / self.queries if self.queries else 0.0}


class NativeRadixPrefixCache:
    """:class:`RadixPrefixCache` backed by the C++ ``_native.RadixCache`` over a
    :class:`~.kv_cache.NativeBlockManager` (same matches and LRU evictions; an eviction is
    O(log n) rather than a walk over the tree)."""

    def __init__(self, blocks):
        self.bm = blocks
        self.bs = blocks.block_size
        from .. import _native

        self.tree = _native.RadixCache(blocks.pool)

    def match(self, tokens: list[int]) -> tuple[list[int], int]:
        blocks, n = self.tree.match(list(tokens))
        return list(blocks), n

    def insert(self, tokens: list[int], block_table: list[int]) -> None:
        self.tree.insert(list(tokens), list(block_table))

    def evict(self, n: int) -> int:
        return self.tree.evict(n)

    @property
    def n_blocks(self) -> int:
        return self.tree.n_blocks

    @property
    def hits(self) -> int:
        return self.tree.hits

    @property
    def queries(self) -> int:
        return self.tree.queries

    def stats(self) -> dict:
        q = self.queries
        return {"cached_blocks": self.n_blocks, "queries": q, "hits": self.hits,
                "hit_rate": self.hits / q if q else 0.0}


def new_prefix_cache(blocks):
    """Radix prefix cache matching the block manager's backend (native pool -> native tree)."""
    from .kv_cache import NativeBlockManager

    return NativeRadixPrefixCache(blocks) if isinstance(blocks, NativeBlockManager) else RadixPrefixCache(blocks)
