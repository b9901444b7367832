"""Paged KV-cache block allocator with automatic prefix caching.

Blocks hold ``block_size`` tokens of every layer's K and V. A full block is identified by a chain hash
of its tokens and all tokens before it, so a new request whose prompt extends an earlier transcript
reuses the cached blocks of that transcript (the TextWorld rollout appends to one growing transcript,
so every request after the first one hits). Freed blocks keep their hash and sit in an LRU list; a
cached block is only recycled when no free uncached block is left.
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Tuple


def block_hash(parent: Optional[int], tokens: Sequence[int]) -> int:
    return hash((parent, tuple(tokens)))


class BlockAllocator:
    def __init__(self, num_blocks: int, block_size: int, enable_prefix_caching: bool = True):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.enable_prefix_caching = enable_prefix_caching
        self.ref = [0] * num_blocks
        self.hash_of: List[Optional[int]] = [None] * num_blocks
        self.cached: Dict[int, int] = {}
        # free blocks, least recently freed first; uncached ones are preferred for allocation
        self.free_uncached: "OrderedDict[int, None]" = OrderedDict((b, None) for b in range(num_blocks))
        self.free_cached: "OrderedDict[int, None]" = OrderedDict()
        self.hits = 0
        self.queries = 0

    @property
    def num_free(self) -> int:
        return len(self.free_uncached) + len(self.free_cached)

    def allocate(self) -> Optional[int]:
        if self.free_uncached:
            b, _ = self.free_uncached.popitem(last=False)
        elif self.free_cached:
            b, _ = self.free_cached.popitem(last=False)
            h = self.hash_of[b]
            if h is not None and self.cached.get(h) == b:
                del self.cached[h]
            self.hash_of[b] = None
        else:
            return None
        self.ref[b] = 1
        return b

    def free(self, blocks: Sequence[int]) -> None:
        for b in blocks:
            self.ref[b] -= 1
            if self.ref[b] == 0:
                if self.hash_of[b] is not None:
                    self.free_cached[b] = None
                else:
                    self.free_uncached[b] = None

    def match_prefix(self, tokens: Sequence[int]) -> Tuple[List[int], List[int]]:
        """Cached full blocks covering a prefix of ``tokens``; returns (blocks, their chain hashes).
        The caller owns a reference to each returned block."""
        if not self.enable_prefix_caching:
            return [], []
        bs = self.block_size
        blocks: List[int] = []
        hashes: List[int] = []
        parent = None
        for i in range(len(tokens) // bs):
            h = block_hash(parent, tokens[i * bs : (i + 1) * bs])
            self.queries += 1
            b = self.cached.get(h)
            if b is None:
                break
            self.hits += 1
            if self.ref[b] == 0:
                self.free_cached.pop(b, None)
            self.ref[b] += 1
            blocks.append(b)
            hashes.append(h)
            parent = h
        return blocks, hashes

    def register(self, block: int, h: int) -> None:
        if not self.enable_prefix_caching:
            return
        if h in self.cached and self.cached[h] != block:
            return  # identical content already cached in another block
        self.hash_of[block] = h
        self.cached[h] = block

    def clear_cache(self) -> None:
        """Forget every cached prefix (weights changed, the cached K/V is stale)."""
        self.cached.clear()
        for b in list(self.free_cached.keys()):
            self.hash_of[b] = None
            self.free_uncached[b] = None
        self.free_cached.clear()
        for b in range(self.num_blocks):
            if self.ref[b] > 0:
                self.hash_of[b] = None
