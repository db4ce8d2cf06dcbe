"""Paged KV block manager with prefix caching.

Blocks hold 16 tokens. A *full* block gets a content hash chained on its parent
(``h_i = H(h_{i-1}, tokens of block i)``) and stays findable by that hash after its
sequences finish (reference count 0 -> LRU of cached blocks) until the allocator
needs it back. Restored AMF pages are registered the same way
(:meth:`register_computed`): once a prefix is restored into blocks, the blocks are
indistinguishable from prefilled ones -- later requests with the same prefix reuse
them from the prefix cache, and eviction treats them like any other cached block.
The reference never reached this state in vLLM v1: its pool writes opaque
``_ExternalBlockRef`` objects that the block manager ignores
(compressed_vram_pool.py:823-885) and its scheduler hook is inert
(decode_scheduler.py:153-170).
"""
from __future__ import annotations

import hashlib
from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

PAGE = 16


def block_hashes(tokens: Sequence[int], n_blocks: Optional[int] = None) -> List[bytes]:
    """Chained 16-byte hashes of the first ``n_blocks`` full blocks of ``tokens``
    (computed natively; equal hashes mean equal whole prefixes)."""
    from .._native_loader import native

    arr = tokens if isinstance(tokens, np.ndarray) else np.asarray(tokens, dtype=np.int64)
    if arr.dtype != np.int32:
        arr = (arr.astype(np.int64) & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
    h = native().block_chain_hashes(arr, PAGE, -1 if n_blocks is None else n_blocks)
    raw = h.tobytes()
    return [raw[16 * i:16 * (i + 1)] for i in range(h.shape[0])]


class BlockManager:
    def __init__(self, num_blocks: int, enable_prefix_cache: bool = True):
        self.num_blocks = num_blocks
        self.enable_prefix_cache = enable_prefix_cache
        self.ref = [0] * num_blocks
        self.hash_of: List[Optional[bytes]] = [None] * num_blocks
        self.by_hash: Dict[bytes, int] = {}
        self.free: List[int] = list(range(num_blocks - 1, -1, -1))  # never-used / hash-free blocks
        self.cached: "OrderedDict[int, None]" = OrderedDict()       # ref 0 but holding a hash (LRU order)
        self.stat_hits = 0
        self.stat_evictions = 0

    # ------------------------------------------------------------------ capacity
    def num_free(self) -> int:
        return len(self.free) + len(self.cached)

    def can_allocate(self, n: int) -> bool:
        return self.num_free() >= n

    # ------------------------------------------------------------------ alloc / free
    def _take(self) -> int:
        if self.free:
            b = self.free.pop()
        elif self.cached:
            b, _ = self.cached.popitem(last=False)  # least recently used cached block
            h = self.hash_of[b]
            if h is not None and self.by_hash.get(h) == b:
                del self.by_hash[h]
            self.hash_of[b] = None
            self.stat_evictions += 1
        else:
            raise MemoryError("KV cache out of blocks")
        self.ref[b] = 1
        return b

    def allocate(self, n: int) -> List[int]:
        if not self.can_allocate(n):
            raise MemoryError(f"KV cache needs {n} blocks, {self.num_free()} free")
        return [self._take() for _ in range(n)]

    def match_prefix(self, hashes: Sequence[bytes]) -> List[int]:
        """Longest run of cached blocks for the given chain; takes a reference on each."""
        if not self.enable_prefix_cache:
            return []
        got: List[int] = []
        for h in hashes:
            b = self.by_hash.get(h)
            if b is None:
                break
            if self.ref[b] == 0:
                self.cached.pop(b, None)
            self.ref[b] += 1
            got.append(b)
        self.stat_hits += len(got)
        return got

    def register_computed(self, blocks: Sequence[int], hashes: Sequence[bytes]) -> None:
        """Mark full blocks as holding the KV of the given hash chain (after prefill or
        after an AMF restore)."""
        if not self.enable_prefix_cache:
            return
        for b, h in zip(blocks, hashes):
            if self.hash_of[b] == h:
                continue
            if h in self.by_hash and self.by_hash[h] != b:
                continue  # another block already carries this content
            self.hash_of[b] = h
            self.by_hash[h] = b

    def release(self, blocks: Sequence[int]) -> None:
        for b in blocks:
            self.ref[b] -= 1
            if self.ref[b] < 0:
                raise RuntimeError(f"block {b} released twice")
            if self.ref[b] == 0:
                if self.hash_of[b] is not None and self.enable_prefix_cache:
                    self.cached[b] = None
                    self.cached.move_to_end(b)
                else:
                    self.hash_of[b] = None
                    self.free.append(b)

    def evict_cached(self, fraction: float = 1.0) -> int:
        """Drop a fraction of the cached (unreferenced) blocks, oldest first."""
        n = int(len(self.cached) * fraction)
        for _ in range(n):
            b, _ = self.cached.popitem(last=False)
            h = self.hash_of[b]
            if h is not None and self.by_hash.get(h) == b:
                del self.by_hash[h]
            self.hash_of[b] = None
            self.free.append(b)
        self.stat_evictions += n
        return n

    def stats(self) -> Dict[str, int]:
        return {"num_blocks": self.num_blocks, "free": len(self.free), "cached": len(self.cached),
                "in_use": self.num_blocks - len(self.free) - len(self.cached), "prefix_hits": self.stat_hits,
                "evictions": self.stat_evictions}
