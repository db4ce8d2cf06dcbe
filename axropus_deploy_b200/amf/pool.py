"""G1 hot tier: the node-wide KV pool, sharded across the GPUs by prefix key.

Every GPU holds one *shard*: a device slab of fixed-size chunk slots. A chunk holds
one KV page (16 tokens) of a prefix for all layers, K and V, and heads, in the
shard's storage format (``raw`` bf16, ``fp8`` e4m3 with one scale per page and
head, or ``int4`` g64 asymmetric). Which slots belong to which prefix lives in the
native :class:`ShardDirectory` (POSIX shared memory, one robust lock per shard), so
any rank of the node can find, pin and fill any shard without messaging its owner.

Data never leaves the GPUs on the hot path:

* capture -- ``page_transfer(cache -> owner slab)``: the kernel quantises the live
  pages and stores them into the owner's slab. When the owner is another GPU its
  slab is mapped into this process and the stores cross NVLink from inside the
  kernel (fused quantise + push).
* restore -- ``page_transfer(owner slab -> cache)``: loads (over NVLink when the
  owner is remote), dequantises and scatters into this rank's block table in one
  kernel (fused pull + dequantise + scatter).

Reference: CompressedVRAMPool (korith_vllm_ext/compressed_vram_pool.py) -- one
process, one GPU, per-layer slabs with contiguous spans, PyTorch codecs and
index-put scatter. Its public API (get / put_from_raw / put_from_vllm /
restore_to_tensor / restore_to_vllm / delete / clear / map_into_vllm / stats) is
kept on :class:`G1Pool`.
"""
from __future__ import annotations

import logging
import math
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence

import torch

from .._native_loader import native
from ..ops.kvcache import (BF16, INT4, PAGE, POOL_FORMATS, KVCache, PageStore, Side, decode_units, encode_units,
                           meta_unit_bytes, page_transfer, unit_bytes)
from .keys import pool_key, pool_key2, pool_key_int

log = logging.getLogger(__name__)
CHUNK_ALIGN = 256


class PoolSlab(PageStore):
    """One shard's chunk slots. ``buffer`` may be any uint8 tensor (a symmetric-memory
    allocation, a shared-memory file mapping for CPU ranks, or a plain tensor)."""

    def __init__(self, n_slots: int, num_layers: int, num_kv_heads: int, head_dim: int, fmt: str = "raw",
                 device="cpu", buffer: Optional[torch.Tensor] = None):
        self.fmt_name = fmt
        self.fmt = POOL_FORMATS[fmt]
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.n_slots = n_slots
        self.unit = unit_bytes(self.fmt, head_dim)
        self.munit = meta_unit_bytes(self.fmt, head_dim)
        self.n_units = num_layers * 2 * num_kv_heads
        self.data_region = self.n_units * self.unit
        self.chunk = self.chunk_bytes(num_layers, num_kv_heads, head_dim, fmt)
        if buffer is None:
            buffer = torch.zeros(n_slots * self.chunk, dtype=torch.uint8, device=device)
        if buffer.numel() < n_slots * self.chunk:
            raise ValueError("pool buffer smaller than n_slots * chunk")
        self.slab = buffer
        self.device = buffer.device

    @staticmethod
    def chunk_bytes(num_layers: int, num_kv_heads: int, head_dim: int, fmt: str) -> int:
        f = POOL_FORMATS[fmt]
        n = num_layers * 2 * num_kv_heads * (unit_bytes(f, head_dim) + meta_unit_bytes(f, head_dim))
        return (n + CHUNK_ALIGN - 1) // CHUNK_ALIGN * CHUNK_ALIGN

    def side(self, base: Optional[int] = None) -> Side:
        b = self.slab.data_ptr() if base is None else base
        H = self.num_kv_heads
        return Side(b, b + self.data_region if self.munit else 0,
                    (H * self.unit, self.chunk, self.unit, H * self.munit, self.chunk, self.munit), self.fmt)

    def _views(self, ids: torch.Tensor):
        L, H, D = self.num_layers, self.num_kv_heads, self.head_dim
        rows = self.slab[: self.n_slots * self.chunk].view(self.n_slots, self.chunk)[ids.long().to(self.slab.device)]
        d = rows[:, : self.data_region]
        if self.fmt == BF16:
            d = d.contiguous().view(torch.bfloat16).view(-1, L, 2, H, PAGE, D)
        elif self.fmt == INT4:
            d = d.reshape(-1, L, 2, H, PAGE, D // 2)
        else:
            d = d.reshape(-1, L, 2, H, PAGE, D)
        m = None
        if self.munit:
            mb = rows[:, self.data_region: self.data_region + self.n_units * self.munit].contiguous()
            if self.fmt == INT4:
                m = mb.view(torch.float16).view(-1, L, 2, H, PAGE, D // 64, 2)
            else:
                m = mb.view(torch.float32).view(-1, L, 2, H)
        return d, m

    def read_units(self, ids: torch.Tensor) -> torch.Tensor:
        d, m = self._views(ids)
        return decode_units(self.fmt, d, m)

    def write_units(self, ids: torch.Tensor, vals: torch.Tensor) -> None:
        d, m = encode_units(self.fmt, vals)
        rows = self.slab[: self.n_slots * self.chunk].view(self.n_slots, self.chunk)
        n = d.shape[0]
        payload = d.contiguous().view(torch.uint8).reshape(n, -1)
        if m is not None:
            payload = torch.cat((payload, m.contiguous().view(torch.uint8).reshape(n, -1)), dim=1)
        rows[ids.long().to(rows.device), : payload.shape[1]] = payload.to(rows.device)


class DenseStore(PageStore):
    """Pages of one prefix as a dense ``[n_pages, L, 2, H, 16, D]`` bf16 tensor."""

    def __init__(self, pages: torch.Tensor):
        self.t = pages
        self.num_layers, _, self.num_kv_heads, _, self.head_dim = pages.shape[1], pages.shape[2], pages.shape[3], \
            pages.shape[4], pages.shape[5]
        self.fmt = BF16
        self.device = pages.device
        self.unit = PAGE * self.head_dim * 2

    @classmethod
    def from_tokens(cls, kv: torch.Tensor) -> "DenseStore":
        """[L, 2, T, H, D] (T multiple of 16) -> pages."""
        L, _, T, H, D = kv.shape
        n = T // PAGE
        pages = kv[:, :, : n * PAGE].reshape(L, 2, n, PAGE, H, D).permute(2, 0, 1, 4, 3, 5).contiguous()
        return cls(pages.to(torch.bfloat16))

    def to_tokens(self) -> torch.Tensor:
        n, L, _, H, P, D = self.t.shape
        return self.t.permute(1, 2, 0, 4, 3, 5).reshape(L, 2, n * P, H, D)

    def side(self) -> Side:
        H, L = self.num_kv_heads, self.num_layers
        return Side(self.t.data_ptr(), 0, (H * self.unit, L * 2 * H * self.unit, self.unit, 0, 0, 0), BF16)

    def read_units(self, ids: torch.Tensor) -> torch.Tensor:
        return self.t[ids.long().to(self.t.device)].float()

    def write_units(self, ids: torch.Tensor, vals: torch.Tensor) -> None:
        self.t[ids.long().to(self.t.device)] = vals.to(self.t.dtype)


@dataclass
class PoolHit:
    key: str
    shard: int
    slots: torch.Tensor  # int32 [n_pages] slot ids in the owner shard
    n_tokens: int
    pinned: bool = True


@dataclass
class PoolEntryInfo:
    """Reference-style entry view returned by ``G1Pool.get``."""

    prefix_hash: str
    num_layers: int
    num_tokens: int
    format: str
    shard: int
    slots: List[int] = field(default_factory=list)
    hit_count: int = 0

    def nbytes(self) -> int:
        return 0


class G1Pool:
    """This rank's handle on the node-wide sharded G1 pool.

    ``slabs`` lists one PoolSlab per shard: the local one owns its memory; remote ones
    wrap a mapping of the peer's slab (``remote_bases`` gives their device addresses
    when the mapping is not a torch tensor of this process)."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, fmt: str = "raw",
                 slots_per_shard: int = 64, device="cpu", rank: int = 0, world: int = 1,
                 dir_name: str = "", slabs: Optional[List[PoolSlab]] = None,
                 remote_bases: Optional[List[int]] = None, entry_cap: int = 4096, create_dir: bool = True):
        self.num_layers, self.num_kv_heads, self.head_dim = num_layers, num_kv_heads, head_dim
        self.fmt_name = fmt
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.chunk = PoolSlab.chunk_bytes(num_layers, num_kv_heads, head_dim, fmt)
        self.slots_per_shard = slots_per_shard
        if slabs is None:
            slabs = [PoolSlab(slots_per_shard, num_layers, num_kv_heads, head_dim, fmt, device)
                     if s == rank or world == 1 else None for s in range(world)]
        self.slabs = slabs
        self.remote_bases = remote_bases or [0] * world
        n = native()
        self.dir = n.ShardDirectory(dir_name, world, [slots_per_shard] * world, self.chunk, entry_cap,
                                    attach=not create_dir)
        self._lock = threading.RLock()
        self._known: Dict[str, int] = {}
        self.stat_bytes_restored = 0
        self.stat_restore_s = 0.0

    # ------------------------------------------------------------------ geometry
    def owner(self, key: str) -> int:
        return pool_key_int(key) % self.world

    def shard_side(self, shard: int) -> Side:
        slab = self.slabs[shard]
        if slab is not None:
            return slab.side()
        proto = self._proto()
        return proto.side(base=self.remote_bases[shard])

    def _proto(self) -> PoolSlab:
        for s in self.slabs:
            if s is not None:
                return s
        raise RuntimeError("no local pool slab")

    def store_for(self, shard: int) -> PoolSlab:
        return self.slabs[shard] if self.slabs[shard] is not None else self._proto()

    # ------------------------------------------------------------------ core ops
    def lookup(self, key: str, key2: int = 0, pin: bool = True) -> Optional[PoolHit]:
        shard = self.owner(key)
        r = self.dir.lookup(shard, pool_key_int(key), key2, self.rank if pin else -1)
        if r is None:
            return None
        n_tokens, _fmt, slots = r
        return PoolHit(key, shard, torch.from_numpy(slots.copy()), int(n_tokens), pin)

    def release(self, hit: PoolHit) -> None:
        if hit.pinned:
            self.dir.unpin(hit.shard, pool_key_int(hit.key), self.rank)
            hit.pinned = False

    def contains(self, key: str) -> bool:
        return self.dir.contains(self.owner(key), pool_key_int(key), 0)

    def capture(self, key: str, src: PageStore, src_blocks: torch.Tensor, n_tokens: int, key2: int = 0,
                savings_ms: float = 0.0, sync: bool = True) -> bool:
        """Store the first ``len(src_blocks)`` pages of ``src`` under ``key``."""
        n_pages = int(src_blocks.numel())
        if n_pages == 0:
            return False
        shard = self.owner(key)
        fmt_id = self._proto().fmt
        st, slots, evicted = self.dir.begin_insert(shard, pool_key_int(key), key2, n_pages, n_tokens, fmt_id,
                                                   self.rank, savings_ms)
        name = str(st).split(".")[-1]
        if name == "EXISTS":
            return True
        if name != "OK":
            log.debug("pool capture %s -> shard %d refused: %s", key, shard, name)
            return False
        try:
            dst = self.store_for(shard)
            page_transfer(src, src_blocks, dst, torch.from_numpy(slots.copy()),
                          dst_side=self.shard_side(shard) if self.slabs[shard] is None else None)
            if sync and dst.device.type == "cuda" or (src.device.type == "cuda" and sync):
                torch.cuda.current_stream().synchronize()
        except Exception:
            self.dir.abort(shard, pool_key_int(key))
            raise
        self.dir.commit(shard, pool_key_int(key))
        return True

    def restore(self, hit: PoolHit, dst: PageStore, dst_blocks: torch.Tensor, n_pages: Optional[int] = None) -> int:
        """Pull the hit's pages into ``dst_blocks`` of ``dst``; returns pages restored."""
        n = min(int(hit.slots.numel()), int(dst_blocks.numel()) if n_pages is None else n_pages)
        if n <= 0:
            return 0
        src = self.store_for(hit.shard)
        page_transfer(src, hit.slots[:n], dst, dst_blocks[:n],
                      src_side=self.shard_side(hit.shard) if self.slabs[hit.shard] is None else None)
        return n

    # ------------------------------------------------------------------ reference API
    def __contains__(self, prefix_hash: str) -> bool:
        return self.contains(prefix_hash)

    def __len__(self) -> int:
        return sum(self.dir.info(s)["entries"] for s in range(self.world))

    def num_prefixes(self) -> int:
        return len(self)

    def capacity_bytes(self) -> int:
        return self.world * self.slots_per_shard * self.chunk

    def used_bytes(self) -> int:
        return sum((i["n_slots"] - i["free_slots"]) * self.chunk for i in (self.dir.info(s) for s in range(self.world)))

    def get(self, prefix_hash: str) -> Optional[PoolEntryInfo]:
        hit = self.lookup(prefix_hash, pin=False)
        if hit is None:
            return None
        return PoolEntryInfo(prefix_hash, self.num_layers, hit.n_tokens, self.fmt_name, hit.shard,
                             hit.slots.tolist())

    def put_from_raw(self, prefix_hash: str, raw_kv: torch.Tensor, *, format: Optional[str] = None,
                     savings_ms: float = 0.0) -> bool:
        """Insert a dense ``[L, 2, T, H, D]`` (or ``[L, 2, nb, bs, H, D]``) KV tensor.
        Only whole 16-token pages are stored."""
        if raw_kv.dim() == 6:
            L, _, nb, bs, H, D = raw_kv.shape
            raw_kv = raw_kv.reshape(L, 2, nb * bs, H, D)
        if raw_kv.dim() != 5 or raw_kv.shape[1] != 2:
            raise ValueError(f"put_from_raw: expected [L,2,T,H,D], got {tuple(raw_kv.shape)}")
        T = raw_kv.shape[2]
        n = T // PAGE
        if n == 0:
            return False
        dense = DenseStore.from_tokens(raw_kv.to(self.device))
        return self.capture(prefix_hash, dense, torch.arange(n, dtype=torch.int32), n * PAGE,
                            savings_ms=savings_ms)

    promote_from_raw = put_from_raw

    def restore_to_tensor(self, prefix_hash: str, target_dtype: torch.dtype = torch.bfloat16) -> Optional[torch.Tensor]:
        hit = self.lookup(prefix_hash)
        if hit is None:
            return None
        try:
            n = int(hit.slots.numel())
            dense = DenseStore(torch.empty(n, self.num_layers, 2, self.num_kv_heads, PAGE, self.head_dim,
                                           dtype=torch.bfloat16, device=self.device))
            self.restore(hit, dense, torch.arange(n, dtype=torch.int32))
            if self.device.type == "cuda":
                torch.cuda.current_stream().synchronize()
            return dense.to_tokens()[:, :, : hit.n_tokens].to(target_dtype)
        finally:
            self.release(hit)

    def put_from_vllm(self, prefix_hash: str, gpu_cache: KVCache, block_table: Sequence[int], n_tokens: int, *,
                      format: Optional[str] = None, savings_ms: float = 0.0) -> bool:
        n = min(n_tokens // PAGE, len(block_table))
        return self.capture(prefix_hash, gpu_cache, torch.tensor(list(block_table[:n]), dtype=torch.int32),
                            n * PAGE, savings_ms=savings_ms)

    def restore_to_vllm(self, prefix_hash: str, gpu_cache: KVCache, block_table: Sequence[int]) -> int:
        hit = self.lookup(prefix_hash)
        if hit is None:
            return 0
        try:
            n = self.restore(hit, gpu_cache, torch.tensor(list(block_table), dtype=torch.int32))
            if gpu_cache.device.type == "cuda":
                torch.cuda.current_stream().synchronize()
            return min(hit.n_tokens, n * PAGE)
        finally:
            self.release(hit)

    def delete(self, prefix_hash: str) -> bool:
        return bool(self.dir.remove(self.owner(prefix_hash), pool_key_int(prefix_hash)))

    def clear(self) -> None:
        for s in range(self.world):
            self.dir.clear(s)

    def map_into_vllm(self, prefix_hash: str, seq_id: Any, block_table: Any) -> bool:
        """Write external block references (``is_external=True``) for the prefix's pool
        slots into a dict-of-lists block table (reference: compressed_vram_pool.py:823-885).
        The engine of this framework registers restored pages through its own block
        manager instead; this keeps the reference's hook API working."""
        hit = self.lookup(prefix_hash, pin=False)
        if hit is None:
            return False
        try:
            table = block_table[seq_id]
            for i, slot in enumerate(hit.slots.tolist()):
                ref = {"is_external": True, "shard": hit.shard, "slot": slot}
                if i < len(table):
                    table[i] = ref
                else:
                    table.append(ref)
            return True
        except Exception as exc:
            log.warning("map_into_vllm failed for seq %s: %s", seq_id, exc)
            return False

    def stats(self) -> Dict[str, Any]:
        infos = [self.dir.info(s) for s in range(self.world)]
        return {
            "hits": sum(i["hits"] for i in infos),
            "misses": sum(i["misses"] for i in infos),
            "inserts": sum(i["inserts"] for i in infos),
            "evictions": sum(i["evictions"] for i in infos),
            "bytes_stored": sum(i["bytes_stored"] for i in infos),
            "bytes_evicted": sum(i["bytes_evicted"] for i in infos),
            "num_prefixes": sum(i["entries"] for i in infos),
            "used_bytes": self.used_bytes(),
            "capacity_bytes": self.capacity_bytes(),
            "format": self.fmt_name,
            "shards": infos,
        }


def prefix_keys(tokens: Sequence[int]) -> tuple:
    """(pool key, check hash) for a page-aligned token prefix."""
    return pool_key(tokens), pool_key2(tokens)
