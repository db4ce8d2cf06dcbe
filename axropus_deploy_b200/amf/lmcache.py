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
            t = self._mem.pop(key, None)
            self._pending.pop(key, None)
            if t is None:
                return False
            self._bytes -= t.numel() * t.element_size()
            return True

    def stats(self) -> Dict[str, Any]:
        return dict(self.stat, enabled=self.enabled, backend=self.backend, entries=len(self._mem),
                    bytes=self._bytes, library=self._engine is not None)
