"""Builds this rank's handle on the node-wide sharded G1 pool.

GPU ranks allocate their shard slab in symmetric memory and exchange handles, so
every rank maps every peer's slab; the page-transfer kernel then reads (restore)
or writes (capture) a peer shard with plain loads/stores over NVLink. CPU ranks
(gloo tests) back each shard with a shared-memory file mapped by all ranks.
The shard directory (slot allocator + index) is created by rank 0 in POSIX shared
memory and attached by the others after a barrier.
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch

from ..amf.pool import G1Pool, PoolSlab
from .dist import DistInfo, barrier


def _shm_path(tag: str, shard: int) -> str:
    return f"/dev/shm/{tag}_slab{shard}"


def build_pool(info: DistInfo, num_layers: int, num_kv_heads: int, head_dim: int, fmt: str,
               slots_per_shard: int, tag: str, entry_cap: int = 4096) -> G1Pool:
    chunk = PoolSlab.chunk_bytes(num_layers, num_kv_heads, head_dim, fmt)
    nbytes = slots_per_shard * chunk
    dir_name = f"/{tag}_{fmt}_dir" if info.world > 1 else ""
    slabs: List[Optional[PoolSlab]] = [None] * info.world
    bases = [0] * info.world
    if info.device.type == "cuda":
        if info.world > 1:
            import torch.distributed as dist
            import torch.distributed._symmetric_memory as symm

            buf = symm.empty(nbytes, dtype=torch.uint8, device=info.device)
            buf.zero_()
            hdl = symm.rendezvous(buf, dist.group.WORLD)
            bases = [int(p) for p in hdl.buffer_ptrs]
            slabs[info.rank] = PoolSlab(slots_per_shard, num_layers, num_kv_heads, head_dim, fmt, info.device, buf)
            _keepalive.append((buf, hdl))
        else:
            slabs[0] = PoolSlab(slots_per_shard, num_layers, num_kv_heads, head_dim, fmt, info.device)
    else:
        for s in range(info.world):
            path = _shm_path(tag + "_" + fmt, s)
            if info.rank == s:
                with open(path, "wb") as f:
                    f.truncate(nbytes)
        barrier(info)
        for s in range(info.world):
            t = torch.from_file(_shm_path(tag + "_" + fmt, s), shared=True, size=nbytes, dtype=torch.uint8)
            slabs[s] = PoolSlab(slots_per_shard, num_layers, num_kv_heads, head_dim, fmt, "cpu", t)
    if info.rank == 0:
        pool = G1Pool(num_layers, num_kv_heads, head_dim, fmt, slots_per_shard, info.device, info.rank, info.world,
                      dir_name, slabs, bases, entry_cap, create_dir=True)
        barrier(info)
    else:
        barrier(info)
        pool = G1Pool(num_layers, num_kv_heads, head_dim, fmt, slots_per_shard, info.device, info.rank, info.world,
                      dir_name, slabs, bases, entry_cap, create_dir=False)
    barrier(info)
    return pool


def cleanup_shm(tag: str, world: int, fmt: str) -> None:
    for s in range(world):
        try:
            os.remove(_shm_path(tag + "_" + fmt, s))
        except FileNotFoundError:
            pass


_keepalive: list = []
