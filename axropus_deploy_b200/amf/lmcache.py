"""Lower KV tiers below the G1 pool: CPU memory (G3), NVMe files (G4), remote (G5).

Reference: korith_vllm_ext/lmcache_adapter.py -- uses ``lmcache.engine.LMCacheEngine``
when importable, otherwise an in-process dict (cpu/remote) or ``torch.save`` files
``{path}/{hash}.pt`` (nvme); configured by ``AXROPUS_LMCACHE_{ENABLE,BACKEND,PATH,URL}``.

Here the payload of an entry is the prefix's pages as a dense bf16 tensor
``[n_pages, L, 2, H, 16, D]`` (what :class:`~.pool.DenseStore` wraps), kept in pinned
host memory for the CPU tier so a promotion back to the GPU is one DMA. The NVMe
tier writes ``{path}/{key}.pt`` like the reference. The ``lmcache`` library is not
installed on these boxes; when it is importable it is used as the backend.
"""
from __future__ import annotations

import logging
import os
import threading
import time
from collections import OrderedDict
from typing import Any, Dict, Optional

import torch

from ..config import env_bool, env_str

log = logging.getLogger(__name__)


class PinnedPageArena:
    """One pinned host buffer of page slots handed out as contiguous runs (first fit).

    Pinning host memory is slow (it page-locks every page); doing it per stored prefix
    would stall the serving step for hundreds of milliseconds. The arena is pinned once
    and entries are runs of its slots, so a store is one asynchronous device->host DMA
    and a promotion back to the GPU one host->device DMA."""

    def __init__(self, n_pages: int, page_shape, dtype=torch.bfloat16):
        self.page_shape = tuple(page_shape)
        self.n_pages = n_pages
        self.buf = torch.empty(n_pages, *self.page_shape, dtype=dtype, pin_memory=torch.cuda.is_available())
        self.free = [(0, n_pages)]  # sorted, non-adjacent (start, length) runs

    def alloc(self, n: int) -> Optional[int]:
        for i, (s, ln) in enumerate(self.free):
            if ln >= n:
                if ln == n:
                    self.free.pop(i)
                else:
                    self.free[i] = (s + n, ln - n)
                return s
        return None

    def release(self, start: int, n: int) -> None:
        runs = sorted(self.free + [(start, n)])
        merged = []
        for s, ln in runs:
            if merged and merged[-1][0] + merged[-1][1] == s:
                merged[-1] = (merged[-1][0], merged[-1][1] + ln)
            else:
                merged.append((s, ln))
        self.free = merged


class LMCacheAdapter:
    def __init__(self, enabled: Optional[bool] = None, backend: Optional[str] = None, path: Optional[str] = None,
                 url: Optional[str] = None, max_bytes: int = 32 << 30, lookup_timeout_ms: int = 0):
        self.enabled = env_bool("AXROPUS_LMCACHE_ENABLE", False) if enabled is None else enabled
        self.backend = (backend or env_str("AXROPUS_LMCACHE_BACKEND", "cpu")).lower()
        self.path = path or env_str("AXROPUS_LMCACHE_PATH", "/tmp/axropus_lmcache")
        self.url = url or env_str("AXROPUS_LMCACHE_URL", "")
        self.max_bytes = max_bytes
        self.lookup_timeout_ms = lookup_timeout_ms
        self._mem: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        self._bytes = 0
        self._lock = threading.RLock()
        self._pending: Dict[str, Any] = {}  # key -> CUDA event of an in-flight device->host copy
        self._arena: Optional[PinnedPageArena] = None
        self._runs: Dict[str, tuple] = {}  # key -> (start, n) in the arena
        self._copy_stream = None
        self._engine = None
        self.stat = {"hits": 0, "misses": 0, "stores": 0, "evictions": 0, "errors": 0}
        if self.enabled:
            try:  # pragma: no cover - lmcache is not installed here
                from lmcache.engine import LMCacheEngine  # type: ignore

                self._engine = LMCacheEngine
            except Exception:
                self._engine = None
            if self.backend == "nvme":
                os.makedirs(self.path, exist_ok=True)

    def _file(self, key: str) -> str:
        return os.path.join(self.path, f"{key}.pt")

    def lookup(self, key: str) -> Optional[torch.Tensor]:
        if not self.enabled:
            return None
        t0 = time.monotonic()
        with self._lock:
            try:
                if self.backend == "nvme":
                    f = self._file(key)
                    out = torch.load(f, map_location="cpu", weights_only=True) if os.path.exists(f) else None
                else:
                    out = self._mem.get(key)
                    if out is not None:
                        self._mem.move_to_end(key)
                        ev = self._pending.pop(key, None)
                        if ev is not None:
                            ev.synchronize()
            except Exception as exc:
                self.stat["errors"] += 1
                log.warning("LMCache lookup failed for %s: %s", key, exc)
                return None
        if self.lookup_timeout_ms and (time.monotonic() - t0) * 1e3 > self.lookup_timeout_ms:
            self.stat["errors"] += 1
            return None
        self.stat["hits" if out is not None else "misses"] += 1
        return out

    def reserve(self, page_shape, dtype=torch.bfloat16) -> None:
        """Pin the CPU tier's memory once, as slots of ``page_shape`` (one KV page of every
        layer: ``[L, 2, H, 16, D]``), instead of per store."""
        if not self.enabled or self.backend != "cpu" or self._arena is not None:
            return
        page_bytes = int(torch.tensor([], dtype=dtype).element_size())
        for d in page_shape:
            page_bytes *= int(d)
        n = max(1, self.max_bytes // page_bytes)
        self._arena = PinnedPageArena(n, page_shape, dtype)

    def _drop(self, key: str) -> None:
        t = self._mem.pop(key, None)
        self._pending.pop(key, None)
        run = self._runs.pop(key, None)
        if run is not None:
            self._arena.release(*run)
        if t is not None:
            self._bytes -= t.numel() * t.element_size()

    def _store_arena(self, key: str, pages: torch.Tensor) -> bool:
        n = pages.shape[0]
        if n > self._arena.n_pages:
            return False
        if key in self._mem:
            self._drop(key)
        start = self._arena.alloc(n)
        while start is None and self._mem:
            self._drop(next(iter(self._mem)))  # least recently used
            self.stat["evictions"] += 1
            start = self._arena.alloc(n)
        if start is None:
            return False
        view = self._arena.buf[start:start + n]
        if pages.is_cuda:
            # the PCIe copy runs on a side stream so the serving stream does not wait for it
            if self._copy_stream is None:
                self._copy_stream = torch.cuda.Stream(device=pages.device)
            side = self._copy_stream
            side.wait_stream(torch.cuda.current_stream(pages.device))
            with torch.cuda.stream(side):
                view.copy_(pages, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(side)
            pages.record_stream(side)
            self._pending[key] = ev
        else:
            view.copy_(pages)
        self._mem[key] = view
        self._runs[key] = (start, n)
        self._bytes += view.numel() * view.element_size()
        return True

    def contains(self, key: str) -> bool:
        if not self.enabled:
            return False
        if self.backend == "nvme":
            return os.path.exists(self._file(key))
        return key in self._mem

    def store(self, key: str, pages: torch.Tensor) -> bool:
        if not self.enabled:
            return False
        pages = pages.detach()
        with self._lock:
            try:
                if self.backend == "nvme":
                    tmp = self._file(key) + ".tmp"
                    torch.save(pages.cpu(), tmp)
                    os.replace(tmp, self._file(key))
                elif self._arena is not None and tuple(pages.shape[1:]) == self._arena.page_shape:
                    if not self._store_arena(key, pages):
                        self.stat["errors"] += 1
                        return False
                else:
                    if pages.device.type == "cpu":
                        host = pages
                    else:
                        # asynchronous device->host copy into pinned memory (the caching host
                        # allocator reuses blocks); a lookup waits for the copy's event
                        host = torch.empty(pages.shape, dtype=pages.dtype, pin_memory=True)
                        host.copy_(pages, non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record()
                        self._pending[key] = ev
                    n = host.numel() * host.element_size()
                    if key in self._mem:
                        old = self._mem.pop(key)
                        self._bytes -= old.numel() * old.element_size()
                    while self._mem and self._bytes + n > self.max_bytes:
                        old_key, ev = self._mem.popitem(last=False)
                        self._pending.pop(old_key, None)
                        self._bytes -= ev.numel() * ev.element_size()
                        self.stat["evictions"] += 1
                    self._mem[key] = host
                    self._bytes += n
                self.stat["stores"] += 1
                return True
            except Exception as exc:
                self.stat["errors"] += 1
                log.warning("LMCache store failed for %s: %s", key, exc)
                return False

    def evict(self, key: str) -> bool:
        with self._lock:
            if self.backend == "nvme":
                try:
                    os.remove(self._file(key))
                    return True
                except FileNotFoundError:
                    return False
            if key not in self._mem:
                return False
            self._drop(key)
            return True

    def stats(self) -> Dict[str, Any]:
        return dict(self.stat, enabled=self.enabled, backend=self.backend, entries=len(self._mem),
                    bytes=self._bytes, library=self._engine is not None)
