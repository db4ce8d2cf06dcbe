"""Tiered cache router: G1 pool -> LMCache tiers -> cold, with miss reasons, write
policy, promotion and background prefetch.

Same surface as the reference's TieredCacheRouter (korith_vllm_ext/tiered_router.py:
``lookup / store_after_prefill / prefetch / set_prefetch_resolver / stop_prefetch /
stats``, enums ``CacheTier``, ``MissReason``, ``WritePolicy``, ``compute_prefix_hash``),
over this framework's sharded G1 pool. KV payloads crossing this API are dense
``[L, 2, T, H, D]`` tensors, as in the reference; the engine's hot path does not use
them (it moves pages kernel-to-kernel through :class:`~.manager.AmfManager`).
"""
from __future__ import annotations

import enum
import logging
import queue
import threading
import time
from dataclasses import dataclass
from typing import Any, Callable, Dict, Optional, Sequence, Tuple

import torch

from .keys import pool_key
from .lmcache import LMCacheAdapter
from .pool import DenseStore, G1Pool

log = logging.getLogger(__name__)


class CacheTier(enum.Enum):
    G1_AMF = "amf"
    G3_LMCACHE = "lmcache"
    COLD = "cold"


class MissReason(enum.Enum):
    FIRST_REQUEST = "first_request"
    EVICTED_FROM_AMF = "evicted_from_amf"
    LMCACHE_DISABLED = "lmcache_disabled"
    LMCACHE_MISS = "lmcache_miss"
    LMCACHE_ERROR = "lmcache_error"
    FORMAT_MISMATCH = "format_mismatch"
    PREFIX_TOO_SHORT = "prefix_too_short"


class WritePolicy(enum.Enum):
    ALWAYS = "always"
    LARGE_ONLY = "large_only"
    ON_EVICTION = "on_eviction"
    NEVER = "never"


@dataclass
class LookupResult:
    prefix_hash: str
    tier: CacheTier
    payload: Any
    latency_ms: float = 0.0
    miss_reason: Optional[MissReason] = None


def compute_prefix_hash(token_ids: Sequence[int]) -> str:
    """sha256 over little-endian int32 token ids, first 16 hex characters."""
    return pool_key(token_ids)


class TieredCacheRouter:
    def __init__(self, pool: G1Pool, lmcache: Optional[LMCacheAdapter] = None, *, min_prefix_tokens: int = 64,
                 write_policy: WritePolicy = WritePolicy.LARGE_ONLY, large_write_threshold: int = 2048):
        self.pool = pool
        self.lmcache = lmcache or LMCacheAdapter()
        self.min_prefix_tokens = min_prefix_tokens
        self.write_policy = write_policy if isinstance(write_policy, WritePolicy) else WritePolicy(write_policy)
        self.large_write_threshold = large_write_threshold
        self._seen: set = set()
        self._miss = {r: 0 for r in MissReason}
        self._hits = {t: 0 for t in CacheTier}
        self._lat = {t: 0.0 for t in CacheTier}
        self._lock = threading.RLock()
        self._pq: "queue.PriorityQueue[Tuple[int, int, str, Any]]" = queue.PriorityQueue()
        self._pq_seq = 0
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self._resolver: Optional[Callable[[str], Optional[torch.Tensor]]] = None

    # ------------------------------------------------------------------ lookup
    def _record(self, tier: CacheTier, t0: float) -> float:
        lat = (time.monotonic() - t0) * 1e3
        with self._lock:
            self._hits[tier] += 1
            self._lat[tier] += lat
        return lat

    def _miss_result(self, key: str, reason: MissReason, t0: float) -> LookupResult:
        with self._lock:
            if reason in (MissReason.LMCACHE_MISS, MissReason.LMCACHE_DISABLED):
                reason = MissReason.EVICTED_FROM_AMF if key in self._seen else MissReason.FIRST_REQUEST
            self._miss[reason] += 1
        return LookupResult(key, CacheTier.COLD, None, self._record(CacheTier.COLD, t0), reason)

    def note_miss(self, key: str, reason: MissReason) -> MissReason:
        """Count a miss decided outside ``lookup`` (e.g. the engine's token-level probe)."""
        return self._miss_result(key, reason, time.monotonic()).miss_reason

    def lookup(self, prefix_hash: str, token_ids: Optional[Sequence[int]] = None) -> LookupResult:
        t0 = time.monotonic()
        if token_ids is not None and len(token_ids) < self.min_prefix_tokens:
            return self._miss_result(prefix_hash, MissReason.PREFIX_TOO_SHORT, t0)
        entry = self.pool.get(prefix_hash)
        if entry is not None:
            with self._lock:
                self._seen.add(prefix_hash)
            return LookupResult(prefix_hash, CacheTier.G1_AMF, entry, self._record(CacheTier.G1_AMF, t0))
        if not self.lmcache.enabled:
            return self._miss_result(prefix_hash, MissReason.LMCACHE_DISABLED, t0)
        try:
            kv = self.lmcache.lookup(prefix_hash)
        except Exception as exc:  # pragma: no cover - backend specific
            log.warning("LMCache lookup failed: %s", exc)
            return self._miss_result(prefix_hash, MissReason.LMCACHE_ERROR, t0)
        if kv is None:
            return self._miss_result(prefix_hash, MissReason.LMCACHE_MISS, t0)
        self._promote(prefix_hash, kv)
        with self._lock:
            self._seen.add(prefix_hash)
        return LookupResult(prefix_hash, CacheTier.G3_LMCACHE, kv, self._record(CacheTier.G3_LMCACHE, t0))

    # ------------------------------------------------------------------ store
    def should_mirror(self, n_tokens: int, is_eviction: bool = False) -> bool:
        p = self.write_policy
        if p == WritePolicy.NEVER:
            return False
        if p == WritePolicy.ALWAYS:
            return True
        if p == WritePolicy.LARGE_ONLY:
            return n_tokens >= self.large_write_threshold
        return is_eviction

    def store_after_prefill(self, prefix_hash: str, token_ids: Sequence[int], kv: torch.Tensor, *,
                            savings_ms: float = 0.0, format: Optional[str] = None) -> bool:
        with self._lock:
            self._seen.add(prefix_hash)
        ok = self.pool.put_from_raw(prefix_hash, kv, savings_ms=savings_ms)
        if self.should_mirror(len(token_ids)):
            try:
                self.lmcache.store(prefix_hash, DenseStore.from_tokens(kv.detach()).t)
            except Exception as exc:  # pragma: no cover
                log.warning("LMCache store failed: %s", exc)
        return ok

    def on_pool_eviction(self, prefix_hash: str, pages: torch.Tensor) -> None:
        """Mirror an entry leaving G1 into the lower tier (write policy ``on_eviction``)."""
        if self.should_mirror(pages.shape[0] * 16, is_eviction=True):
            self.lmcache.store(prefix_hash, pages)

    def _promote(self, prefix_hash: str, kv: torch.Tensor) -> None:
        try:
            pages = kv if kv.dim() == 6 else DenseStore.from_tokens(kv).t
            dense = DenseStore(pages.to(self.pool.device, non_blocking=True))
            n = pages.shape[0]
            self.pool.capture(prefix_hash, dense, torch.arange(n, dtype=torch.int32), n * 16)
        except Exception as exc:  # pragma: no cover
            log.warning("promotion from lower tier failed: %s", exc)

    # ------------------------------------------------------------------ prefetch
    def set_prefetch_resolver(self, resolver: Callable[[str], Optional[torch.Tensor]]) -> None:
        self._resolver = resolver

    def prefetch(self, prefix_hash: str, priority: int = 0, hint: Any = None) -> None:
        with self._lock:
            self._pq_seq += 1
            seq = self._pq_seq
        self._pq.put((priority, seq, prefix_hash, hint))
        if self._thread is None or not self._thread.is_alive():
            self._stop.clear()
            self._thread = threading.Thread(target=self._prefetch_loop, name="amf-prefetch", daemon=True)
            self._thread.start()

    def stop_prefetch(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=1.0)
            self._thread = None

    def _prefetch_loop(self) -> None:
        while not self._stop.is_set():
            try:
                _, _, key, _ = self._pq.get(timeout=0.2)
            except queue.Empty:
                continue
            try:
                if key in self.pool:
                    continue
                kv = self._resolver(key) if self._resolver is not None else None
                if kv is None and self.lmcache.enabled:
                    kv = self.lmcache.lookup(key)
                if kv is not None:
                    self._promote(key, kv)
            except Exception as exc:  # pragma: no cover
                log.warning("prefetch of %s failed: %s", key, exc)

    # ------------------------------------------------------------------ telemetry
    def stats(self) -> Dict[str, Any]:
        with self._lock:
            return {
                "tier_hits": {t.value: n for t, n in self._hits.items()},
                "tier_latency": {t.value: self._lat[t] / max(1, self._hits[t]) for t in CacheTier},
                "miss_reasons": {r.value: n for r, n in self._miss.items()},
                "pool_stats": self.pool.stats(),
                "lmcache_stats": self.lmcache.stats(),
                "write_policy": self.write_policy.value,
            }

    def log_summary(self) -> None:
        s = self.stats()["tier_hits"]
        tot = max(1, sum(s.values()))
        log.info("[TieredRouter] total=%d amf=%.2f%% lmcache=%.2f%% cold=%.2f%% policy=%s", sum(s.values()),
                 100 * s["amf"] / tot, 100 * s["lmcache"] / tot, 100 * s["cold"] / tot, self.write_policy.value)
