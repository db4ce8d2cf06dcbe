"""AMF manager: the engine-facing tier stack and the ``amf_save_kv`` /
``amf_restore_kv`` worker API.

Lookup order (the reference README's stack, README.md:186-200):

1. G2 live prefix cache -- done by the engine's block manager before calling here;
2. G1 hot tier -- the raw bf16 VRAM cache (``KORITH_VRAM_CACHE_GB``) and/or the
   compressed FP8/INT4 pool (``KORITH_VRAM_POOL_GB`` + ``KORITH_VRAM_POOL_QUANT``),
   both sharded across the node's GPUs;
3. LMCache CPU/NVMe tiers (``AXROPUS_LMCACHE_FALLBACK``), promoted into G1 on a hit
   (``AXROPUS_PROMOTE_LMCACHE_HITS``);
4. the AMF disk store (AMFK files, survives restarts), also promoted;
5. cold prefill.

A hit is matched at page granularity: the probe tries every prefix length that some
G1 entry has (longest first), so a request whose prompt is a stored prefix plus a new
suffix restores the prefix and prefills only the suffix.
"""
from __future__ import annotations

import logging
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence

import numpy as np
import torch

from ..ops.kvcache import PAGE, KVCache, page_transfer
from .disk import DiskTier
from .keys import pool_key, pool_key2
from .lmcache import LMCacheAdapter
from .pool import DenseStore, G1Pool, PoolHit
from .router import MissReason, TieredCacheRouter, WritePolicy

log = logging.getLogger(__name__)


@dataclass
class AmfHit:
    tier: str                 # "g1_raw" | "g1_pool" | "lmcache" | "disk"
    n_tokens: int
    key: str
    pool: Optional[G1Pool] = None
    pool_hit: Optional[PoolHit] = None
    dense: Optional[torch.Tensor] = None  # [n, L, 2, H, 16, D] for lower tiers
    disk_entry: Optional[dict] = None
    lookup_ms: float = 0.0

    @property
    def n_pages(self) -> int:
        return self.n_tokens // PAGE

    def restore(self, cache: KVCache, blocks: torch.Tensor, first_page: int = 0) -> int:
        """Write pages [first_page, n_pages) of the hit into ``blocks`` (one id per page)."""
        n = self.n_pages - first_page
        if n <= 0:
            return 0
        if self.pool_hit is not None:
            slots = self.pool_hit.slots[first_page:first_page + n]
            page_transfer(self.pool.store_for(self.pool_hit.shard), slots, cache, blocks[:n],
                          src_side=self.pool.shard_side(self.pool_hit.shard)
                          if self.pool.slabs[self.pool_hit.shard] is None else None)
            return n
        dense = DenseStore(self.dense.to(cache.device, non_blocking=True))
        page_transfer(dense, torch.arange(first_page, first_page + n, dtype=torch.int32), cache, blocks[:n])
        return n

    def release(self) -> None:
        if self.pool_hit is not None and self.pool is not None:
            self.pool.release(self.pool_hit)


class AmfManager:
    def __init__(self, *, raw_pool: Optional[G1Pool] = None, comp_pool: Optional[G1Pool] = None,
                 lmcache: Optional[LMCacheAdapter] = None, disk: Optional[DiskTier] = None,
                 min_tokens: int = 64, vram_first: bool = True, sync_save: bool = False,
                 lmcache_fallback: bool = False, promote_lmcache_hits: bool = True,
                 lmcache_write_through: bool = False, write_policy: str = "large_only",
                 large_write_threshold: int = 2048, disable_restore: bool = False):
        self.raw_pool = raw_pool
        self.comp_pool = comp_pool
        self.lmcache = lmcache or LMCacheAdapter(enabled=False)
        self.disk = disk
        self.min_tokens = min_tokens
        self.vram_first = vram_first
        self.sync_save = sync_save
        self.lmcache_fallback = lmcache_fallback and self.lmcache.enabled
        self.promote_lmcache_hits = promote_lmcache_hits
        self.lmcache_write_through = lmcache_write_through
        self.disable_restore = disable_restore
        self.capture_enabled = True  # cache admission switch (the policy layer turns it off under negative ROI)
        g1 = raw_pool or comp_pool
        if g1 is not None and self.lmcache.enabled and torch.cuda.is_available() and \
                str(getattr(g1, "device", "cpu")).startswith("cuda"):
            self.lmcache.reserve((g1.num_layers, 2, g1.num_kv_heads, PAGE, g1.head_dim))
        self.router = TieredCacheRouter(g1, self.lmcache, min_prefix_tokens=min_tokens,
                                        write_policy=WritePolicy(write_policy),
                                        large_write_threshold=large_write_threshold) if g1 is not None else None
        self.stat: Dict[str, float] = {"lookups": 0, "hits_g1_raw": 0, "hits_g1_pool": 0, "hits_lmcache": 0,
                                        "hits_disk": 0, "misses": 0, "captures": 0, "capture_failures": 0,
                                        "tokens_restored": 0, "restore_ms": 0.0, "disk_saves": 0}

    @property
    def pools(self) -> List[G1Pool]:
        return [p for p in (self.raw_pool, self.comp_pool) if p is not None]

    # ------------------------------------------------------------------ lookup
    def lookup(self, tokens: Sequence[int], max_tokens: Optional[int] = None) -> Optional[AmfHit]:
        """Longest stored page-aligned prefix of ``tokens[:max_tokens]``."""
        t0 = time.perf_counter()
        self.stat["lookups"] += 1
        limit = len(tokens) if max_tokens is None else min(max_tokens, len(tokens))
        limit = limit // PAGE * PAGE
        if limit < self.min_tokens or self.disable_restore:
            if self.router is not None:
                self.router.note_miss(pool_key(tokens[:limit]) if limit else "", MissReason.PREFIX_TOO_SHORT)
            self.stat["misses"] += 1
            return None
        order = self.pools if self.vram_first else []
        for tier, pool in zip(("g1_raw", "g1_pool"), (self.raw_pool, self.comp_pool)):
            if pool is None or pool not in order:
                continue
            for L in pool.dir.lengths():
                if L > limit or L < self.min_tokens:
                    continue
                t = tokens[:L]
                key = pool_key(t)
                hit = pool.lookup(key, key2=pool_key2(t), pin=True)
                if hit is not None:
                    self.stat["hits_" + tier] += 1
                    return AmfHit(tier, hit.n_tokens, key, pool, hit, lookup_ms=(time.perf_counter() - t0) * 1e3)
        # lower tiers
        if self.lmcache_fallback:
            key = pool_key(tokens[:limit])
            pages = self.lmcache.lookup(key)
            if pages is not None:
                self.stat["hits_lmcache"] += 1
                return AmfHit("lmcache", pages.shape[0] * PAGE, key, dense=pages,
                              lookup_ms=(time.perf_counter() - t0) * 1e3)
        if self.disk is not None and self.disk.enabled:
            reason, entry = self.disk.lookup(np.asarray(tokens[:limit]))
            if entry is not None:
                got = self.disk.load(entry)
                if got is not None:
                    _, pages = got
                    self.stat["hits_disk"] += 1
                    return AmfHit("disk", pages.shape[0] * PAGE, pool_key(tokens[:pages.shape[0] * PAGE]),
                                  dense=pages, disk_entry=entry, lookup_ms=(time.perf_counter() - t0) * 1e3)
            else:
                self.disk.store.note_miss()
        self.stat["misses"] += 1
        if self.router is not None:
            self.router.note_miss(pool_key(tokens[:limit]), MissReason.LMCACHE_MISS)
        return None

    def note_restored(self, hit: AmfHit, restore_ms: float, saved_ms: float) -> None:
        self.stat["tokens_restored"] += hit.n_tokens
        self.stat["restore_ms"] += restore_ms
        if hit.disk_entry is not None and self.disk is not None:
            self.disk.note_hit(hit.disk_entry, hit.n_tokens, restore_ms, saved_ms)
        if hit.pool_hit is not None:
            hit.pool.dir.note_savings(hit.pool_hit.shard, int(hit.key, 16) or 1, saved_ms)

    # ------------------------------------------------------------------ capture
    def target_pool(self) -> Optional[G1Pool]:
        return self.raw_pool if self.raw_pool is not None else self.comp_pool

    def capture(self, tokens: Sequence[int], cache: KVCache, blocks: torch.Tensor, savings_ms: float = 0.0,
                promote_from: Optional[str] = None) -> bool:
        """Save the pages of ``tokens`` (a page-aligned prefix held in ``blocks``) into the
        hot tier, and mirror to LMCache / the disk store according to policy."""
        n = len(tokens) // PAGE
        if n * PAGE < self.min_tokens or n == 0 or not self.capture_enabled:
            return False
        t = tokens[:n * PAGE]
        key = pool_key(t)
        pool = self.target_pool()
        ok = False
        if pool is not None:
            ok = pool.capture(key, cache, blocks[:n], n * PAGE, key2=pool_key2(t), savings_ms=savings_ms)
            self.stat["captures" if ok else "capture_failures"] += 1
        mirror_lm = self.lmcache.enabled and (self.lmcache_write_through or
                                              (self.router is not None and self.router.should_mirror(n * PAGE)))
        want_disk = self.disk is not None and self.disk.enabled and (self.sync_save or pool is None)
        if (mirror_lm and promote_from != "lmcache") or (want_disk and promote_from != "disk"):
            dense = DenseStore(torch.empty(n, cache.num_layers, 2, cache.num_kv_heads, PAGE, cache.head_dim,
                                           dtype=torch.bfloat16, device=cache.device))
            page_transfer(cache, blocks[:n], dense, torch.arange(n, dtype=torch.int32))
            if mirror_lm and promote_from != "lmcache":
                self.lmcache.store(key, dense.t)
            if want_disk and promote_from != "disk":
                try:
                    if self.disk.save(t, dense.t, saved_ms=savings_ms):
                        self.stat["disk_saves"] += 1
                except OSError as exc:  # a full or failing disk loses the mirror copy, never the step
                    self.stat["disk_save_failures"] = self.stat.get("disk_save_failures", 0) + 1
                    log.warning("AMF disk save failed: %s", exc)
        return ok

    # ------------------------------------------------------------------ telemetry
    def stats(self) -> Dict[str, Any]:
        out: Dict[str, Any] = dict(self.stat)
        if self.router is not None:
            out["router"] = self.router.stats()
        if self.disk is not None:
            out["disk"] = self.disk.stats()
        return out
