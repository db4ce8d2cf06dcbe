"""Owner-affinity routing of requests over the data-parallel GPUs of one node.

The G1 pool is sharded over the GPUs by prefix hash (``G1Pool.owner``). A request whose
prefix is pooled is cheapest on the GPU that owns that shard: the restore is a local
copy (≈2.8 TB/s) instead of a pull over NVLink (≈0.75 TB/s), and requests for the same
prefix land on the same GPU, where they share its live prefix-cache pages (and the
shared-prefix decode reads those pages once per step). A capture of a cold prefix is a
local write on its owner as well.

:func:`route_wave` assigns one wave of requests with a per-GPU cap, so every GPU gets
the same amount of work (weak scaling):

* cold requests (no pooled prefix) are spread first, at most one apart per GPU, each on
  its owner when the owner is among the least cold-loaded GPUs (their prefill dominates
  a wave's time, so their count per GPU is what must balance);
* pooled requests go to their owner while it has room, in order; the rest ("routing
  misses") go to the least-loaded GPU and are restored over NVLink from the owner.

The assignment is a pure function of its inputs, so every rank computes the same one
from the same request stream with no communication. Reference counterpart: the
cluster router's AMF-locality placement (platform/runtime/cluster_router.py:408-737),
here for the GPUs of one node.
"""
from __future__ import annotations

from typing import List, Optional, Sequence


def route_wave(owners: Sequence[int], cold: Sequence[bool], world: int, per_rank: int,
               cold_carry: Optional[List[int]] = None) -> List[int]:
    """owners[i]: shard owner of request i's prefix; cold[i]: no pooled prefix expected.
    Returns the GPU of each request; every GPU gets at most ``per_rank`` (callers pass
    len(owners) / world for an even wave). ``cold_carry`` (one count per GPU, updated in
    place) carries the cold prefills of earlier waves: when a wave's cold requests do not
    divide evenly, the extra ones go to the GPUs with the fewest so far, so over a run of
    waves no GPU collects every remainder (the slowest GPU sets a data-parallel step)."""
    n = len(owners)
    if world <= 1:
        return [0] * n
    if per_rank * world < n:
        raise ValueError("route_wave: per_rank * world must cover the wave")
    load = [0] * world
    cold_load = [0] * world
    carry = cold_carry if cold_carry is not None else [0] * world
    out = [-1] * n

    def least(keys) -> int:
        return min(range(world), key=lambda r: (keys(r), r))

    for i in range(n):
        if not cold[i]:
            continue
        o = owners[i] % world
        best = min((cold_load[q], carry[q]) for q in range(world) if load[q] < per_rank)
        if (cold_load[o], carry[o]) == best and load[o] < per_rank:
            r = o
        else:
            r = least(lambda q: (load[q] >= per_rank, cold_load[q], carry[q], load[q]))
        out[i] = r
        load[r] += 1
        cold_load[r] += 1
    for q in range(world):
        carry[q] += cold_load[q]
    for i in range(n):
        if cold[i]:
            continue
        o = owners[i] % world
        r = o if load[o] < per_rank else least(lambda q: (load[q] >= per_rank, load[q]))
        out[i] = r
        load[r] += 1
    return out


def routing_stats(owners: Sequence[int], cold: Sequence[bool], assigned: Sequence[int]) -> dict:
    """Share of pooled requests served away from their owner (NVLink restores)."""
    hits = [i for i in range(len(owners)) if not cold[i]]
    miss = sum(1 for i in hits if assigned[i] != owners[i])
    return {"pooled": len(hits), "routing_misses": miss, "miss_share": miss / len(hits) if hits else 0.0}
