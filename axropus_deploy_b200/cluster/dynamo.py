"""Integration with a disaggregated serving frontend of the Dynamo kind: a KV-aware
worker-scoring plugin, a block storage backend that keeps whole-prefix snapshots, and an
event subscriber that persists valuable evicted prefixes.

Cost model (B200, measured by this framework, not extrapolated from other hardware):
cold prefill of Llama-3-8B is ~65 K tokens/s at 8 K context with attention growing
linearly in the context (:func:`prefill_ms`); a restore moves the KV at the rate of the
tier it comes from (:data:`TIER_GBPS`: G1 pool in HBM, pinned host memory, NVMe,
another node) plus a fixed launch cost (:func:`restore_ms`). Both take the model's KV
bytes per token, so other models are priced by their own footprint.

* :class:`AmfRouterPlugin` -- ``score_workers(request_tokens, prefix_hash, tenant,
  candidates)``: per worker ``kv_overlap * w_kv + restore_saving * w_restore - load *
  w_load``, where ``restore_saving`` is the fraction of the prefill a restore from the
  worker's best AMF tier removes; below ``min_prefix_tokens`` (default 4096) only the
  frontend's overlap and load count. Weights from ``AMF_KV_OVERLAP_WEIGHT`` (0.5),
  ``AMF_RESTORE_WEIGHT`` (0.8), ``AMF_LOAD_WEIGHT`` (0.3).
* :class:`AmfStorageBackend` -- ``register_volume / put / get / delete / stats``: blocks
  put under a prefix are aggregated into one snapshot when the prefix completes (or
  on :meth:`flush`); an admission gate keeps only snapshots whose prefill/restore ratio
  reaches ``min_admit_roi``; a validator refuses a snapshot whose model hash / KV
  version (required) or RoPE / sampling fields (when both sides carry them) differ
  from the request; when the volume is full the entry with the least value
  (saved ms per byte, decayed by age, boosted by hits) is evicted.
* :class:`EventSubscriber` -- consumes KV block events (created / updated / evicted) from
  any iterable or queue (an in-process stand-in for the frontend's message bus), tracks
  prefixes, and on eviction of a prefix long enough to be worth keeping hands it to a
  persist callback (e.g. the AMF coordinator register).

Reference: platform/runtime/dynamo_amf_router.py:56-334, dynamo_nixl_backend.py:61-632,
dynamo_event_subscriber.py:57-513.
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, Iterable, List, Optional, Tuple

LLAMA3_8B_KV_BYTES_PER_TOKEN = 131072
TIER_GBPS = {"vram": 2400.0, "G1": 2400.0, "nvlink": 700.0, "ram": 50.0, "G2": 50.0, "nvme": 7.0, "G3": 7.0,
             "remote": 5.0, "G4": 5.0}


def _envf(name: str, default: float) -> float:
    try:
        return float(os.environ.get(name, "") or default)
    except ValueError:
        return default


def prefill_ms(tokens: int, tok_s: float = 65000.0, ctx_ref: int = 8192) -> float:
    """Cold prefill time: linear GEMM cost plus attention cost that grows with the context
    (the rate is quoted at ``ctx_ref`` tokens, where attention is ~15% of the time)."""
    t = max(0, tokens)
    lin = t / tok_s * 1e3 * 0.85
    attn = (t / tok_s * 1e3 * 0.15) * (t / ctx_ref)
    return lin + attn


def restore_ms(tokens: int, tier: str = "vram", kv_bytes_per_token: int = LLAMA3_8B_KV_BYTES_PER_TOKEN) -> float:
    bw = TIER_GBPS.get(tier, TIER_GBPS["remote"])
    return 0.2 + max(0, tokens) * kv_bytes_per_token / (bw * 1e9) * 1e3


@dataclass
class WorkerScore:
    worker_id: str
    node_id: str
    kv_overlap: float
    load: float
    amf_restore_savings_ms: float
    combined_score: float
    routed_by: str
    estimated_restore_ms: float
    estimated_recompute_ms: float


class AmfRouterPlugin:
    def __init__(self, coordinator=None, min_prefix_tokens: Optional[int] = None,
                 kv_bytes_per_token: int = LLAMA3_8B_KV_BYTES_PER_TOKEN):
        self.coord = coordinator
        self.w_kv = _envf("AMF_KV_OVERLAP_WEIGHT", 0.5)
        self.w_restore = _envf("AMF_RESTORE_WEIGHT", 0.8)
        self.w_load = _envf("AMF_LOAD_WEIGHT", 0.3)
        self.min_tokens = int(min_prefix_tokens or _envf("AMF_MIN_PREFIX_TOKENS_FOR_AMF", 4096))
        self.kv_bpt = kv_bytes_per_token
        self.stat = {"queries": 0, "amf_routed": 0, "frontend_routed": 0, "savings_ms": 0.0}

    def _holders(self, prefix_hash: str, tenant: str) -> Dict[str, str]:
        """worker_id -> best tier holding the prefix (coordinator lookup, fail-open)."""
        if self.coord is None:
            return {}
        try:
            locs = self.coord.lookup(prefix_hash, tenant) if hasattr(self.coord, "base") else \
                self.coord.lookup(tenant, prefix_hash)
        except Exception:
            return {}
        out: Dict[str, str] = {}
        rank = list(TIER_GBPS)
        for l in locs:
            wid = l.get("worker_id") or l.get("node_id")
            tier = (l.get("metadata") or {}).get("tier", "ram")
            if wid not in out or rank.index(tier if tier in rank else "remote") < rank.index(out[wid]):
                out[wid] = tier if tier in TIER_GBPS else "remote"
        return out

    def score_workers(self, request_tokens: int, prefix_hash: str, tenant_id: str,
                      candidates: List[Dict[str, Any]]) -> List[WorkerScore]:
        self.stat["queries"] += 1
        use_amf = request_tokens >= self.min_tokens
        holders = self._holders(prefix_hash, tenant_id) if use_amf else {}
        recompute = prefill_ms(request_tokens)
        out = []
        for c in candidates:
            wid = c["worker_id"]
            ov, load = float(c.get("kv_overlap", 0.0)), float(c.get("load", 0.0))
            tier = holders.get(wid) or holders.get(c.get("node_id", ""))
            rest = restore_ms(request_tokens, tier, self.kv_bpt) if tier else recompute
            # what is left to prefill after the frontend's resident overlap
            saving = max(0.0, (recompute - rest) / recompute) if tier and recompute > 0 else 0.0
            saving = max(0.0, saving - ov) if tier else 0.0
            score = ov * self.w_kv + saving * self.w_restore - load * self.w_load
            by = "amf" if saving * self.w_restore > ov * self.w_kv else "frontend"
            out.append(WorkerScore(wid, c.get("node_id", ""), ov, load, (recompute - rest) if tier else 0.0, score,
                                   by, rest if tier else 0.0, recompute))
        out.sort(key=lambda s: s.combined_score, reverse=True)
        if out:
            self.stat["amf_routed" if out[0].routed_by == "amf" else "frontend_routed"] += 1
            self.stat["savings_ms"] += out[0].amf_restore_savings_ms
        return out


class AdmissionGate:
    def __init__(self, min_admit_roi: float = 1.5, kv_bytes_per_token: int = LLAMA3_8B_KV_BYTES_PER_TOKEN):
        self.min_roi = max(0.0, min_admit_roi)
        self.kv_bpt = kv_bytes_per_token
        self.stat = {"admitted": 0, "rejected": 0, "bytes_admitted": 0, "bytes_rejected": 0}

    def evaluate(self, num_tokens: int, tier: str, nbytes: int = 0) -> Tuple[bool, float]:
        roi = prefill_ms(num_tokens) / max(1e-3, restore_ms(num_tokens, tier, self.kv_bpt))
        ok = roi >= self.min_roi
        self.stat["admitted" if ok else "rejected"] += 1
        self.stat["bytes_admitted" if ok else "bytes_rejected"] += nbytes
        return ok, roi


class CorrectnessValidator:
    REQUIRED = ("model_hash", "kv_version")
    OPTIONAL = ("rope_base_bits", "rope_scale_bits", "sampling_hash")

    def __init__(self):
        self.stat = {"pass": 0, "fail": 0}

    def validate(self, stored: Dict[str, Any], request: Dict[str, Any]) -> Tuple[bool, str]:
        for k in self.REQUIRED + self.OPTIONAL:
            a, b = stored.get(k), request.get(k)
            if k in self.OPTIONAL and (a is None or b is None):
                continue
            if a != b:
                self.stat["fail"] += 1
                return False, f"{k} mismatch"
        self.stat["pass"] += 1
        return True, "ok"


@dataclass
class _Snapshot:
    prefix_id: str
    blocks: Dict[str, bytes]
    meta: Dict[str, Any]
    num_tokens: int
    nbytes: int
    saved_ms: float
    created: float = field(default_factory=time.monotonic)
    hits: int = 0

    def value(self, now: float, half_life_s: float = 3600.0) -> float:
        age = max(0.0, now - self.created)
        return self.saved_ms * (1 + self.hits) * 0.5 ** (age / half_life_s) / max(1, self.nbytes)


class AmfStorageBackend:
    def __init__(self, capacity_bytes: int = 0, min_admit_roi: float = 1.5, tier: str = "ram",
                 tokens_per_block: int = 16, kv_bytes_per_token: int = LLAMA3_8B_KV_BYTES_PER_TOKEN):
        self.capacity = capacity_bytes
        self.tier = tier
        self.tpb = tokens_per_block
        self.gate = AdmissionGate(min_admit_roi, kv_bytes_per_token)
        self.validator = CorrectnessValidator()
        self._pending: Dict[str, List[Tuple[str, bytes, Dict[str, Any]]]] = {}
        self._snaps: Dict[str, _Snapshot] = {}
        self._block_to_prefix: Dict[str, str] = {}
        self._mu = threading.Lock()
        self.stat = {"puts": 0, "gets": 0, "hits": 0, "misses": 0, "invalid": 0, "evictions": 0, "snapshots": 0}
        self.registered = False

    def register_volume(self, volume: Dict[str, Any]) -> bool:
        cap = int(volume.get("capacity_bytes", self.capacity) or 0)
        if cap <= 0:
            return False
        self.capacity, self.tier = cap, str(volume.get("tier", self.tier))
        self.registered = True
        return True

    def unregister_volume(self) -> None:
        with self._mu:
            self._snaps.clear()
            self._pending.clear()
            self._block_to_prefix.clear()
        self.registered = False

    def used_bytes(self) -> int:
        return sum(s.nbytes for s in self._snaps.values())

    def put(self, block_id: str, data: bytes, metadata: Dict[str, Any]) -> bool:
        """Buffer a block under ``metadata['prefix_id']``; ``metadata['last']`` completes
        the prefix and turns its blocks into one snapshot."""
        pid = str(metadata.get("prefix_id") or block_id)
        with self._mu:
            self.stat["puts"] += 1
            self._pending.setdefault(pid, []).append((block_id, bytes(data), dict(metadata)))
            if metadata.get("last"):
                return self._flush_locked(pid)
        return True

    def flush(self) -> int:
        with self._mu:
            return sum(int(self._flush_locked(p)) for p in list(self._pending))

    def _flush_locked(self, pid: str) -> bool:
        blocks = self._pending.pop(pid, [])
        if not blocks:
            return False
        ntok = len(blocks) * self.tpb
        nbytes = sum(len(b) for _, b, _ in blocks)
        ok, roi = self.gate.evaluate(ntok, self.tier, nbytes)
        if not ok or nbytes > self.capacity:
            return False
        self._evict_locked(nbytes)
        meta = {k: v for k, v in blocks[0][2].items() if k not in ("last",)}
        saved = prefill_ms(ntok) - restore_ms(ntok, self.tier, self.gate.kv_bpt)
        self._snaps[pid] = _Snapshot(pid, {bid: b for bid, b, _ in blocks}, meta, ntok, nbytes, saved)
        for bid, _, _ in blocks:
            self._block_to_prefix[bid] = pid
        self.stat["snapshots"] += 1
        return True

    def _evict_locked(self, incoming: int) -> None:
        now = time.monotonic()
        while self._snaps and self.used_bytes() + incoming > self.capacity:
            victim = min(self._snaps.values(), key=lambda s: s.value(now))
            for bid in victim.blocks:
                self._block_to_prefix.pop(bid, None)
            del self._snaps[victim.prefix_id]
            self.stat["evictions"] += 1

    def get(self, block_id: str, request_meta: Optional[Dict[str, Any]] = None) -> Optional[bytes]:
        with self._mu:
            self.stat["gets"] += 1
            pid = self._block_to_prefix.get(block_id)
            snap = self._snaps.get(pid) if pid else None
            if snap is None:
                self.stat["misses"] += 1
                return None
            if request_meta is not None:
                ok, _ = self.validator.validate(snap.meta, request_meta)
                if not ok:
                    self.stat["invalid"] += 1
                    return None
            snap.hits += 1
            self.stat["hits"] += 1
            return snap.blocks[block_id]

    def delete(self, block_id: str) -> bool:
        with self._mu:
            pid = self._block_to_prefix.pop(block_id, None)
            snap = self._snaps.get(pid) if pid else None
            if snap is None:
                return False
            snap.blocks.pop(block_id, None)
            snap.nbytes = sum(len(b) for b in snap.blocks.values())
            if not snap.blocks:
                del self._snaps[pid]
            return True

    def stats(self) -> Dict[str, Any]:
        return dict(self.stat, used_bytes=self.used_bytes(), capacity_bytes=self.capacity,
                    admission=dict(self.gate.stat), validator=dict(self.validator.stat), entries=len(self._snaps))


@dataclass
class KvBlockEvent:
    kind: str            # created | updated | evicted
    worker_id: str
    prefix_hash: str
    num_tokens: int
    tier: str = "G1"
    ts: float = field(default_factory=time.time)


class EventSubscriber:
    """Tracks prefixes from block events; persists evicted prefixes worth keeping."""

    def __init__(self, persist: Callable[[Dict[str, Any]], bool], min_tokens: int = 4096, min_saved_ms: float = 20.0):
        self.persist = persist
        self.min_tokens = min_tokens
        self.min_saved_ms = min_saved_ms
        self.prefixes: Dict[Tuple[str, str], Dict[str, Any]] = {}
        self.stat = {"events": 0, "evictions": 0, "persisted": 0, "skipped": 0, "persist_errors": 0}

    def handle(self, ev: KvBlockEvent) -> bool:
        self.stat["events"] += 1
        key = (ev.worker_id, ev.prefix_hash)
        if ev.kind in ("created", "updated"):
            st = self.prefixes.setdefault(key, {"worker_id": ev.worker_id, "prefix_hash": ev.prefix_hash,
                                                "num_tokens": 0, "tier": ev.tier, "first_seen": ev.ts})
            st["num_tokens"] = max(st["num_tokens"], ev.num_tokens)
            st["tier"] = ev.tier
            return False
        if ev.kind != "evicted":
            return False
        self.stat["evictions"] += 1
        st = self.prefixes.pop(key, {"worker_id": ev.worker_id, "prefix_hash": ev.prefix_hash,
                                     "num_tokens": ev.num_tokens, "tier": ev.tier})
        n = max(st["num_tokens"], ev.num_tokens)
        saved = prefill_ms(n) - restore_ms(n, "ram")
        if n < self.min_tokens or saved < self.min_saved_ms:
            self.stat["skipped"] += 1
            return False
        try:
            ok = bool(self.persist(dict(st, num_tokens=n, saved_ms=saved)))
        except Exception:
            self.stat["persist_errors"] += 1
            return False
        self.stat["persisted" if ok else "skipped"] += 1
        return ok

    def run(self, events: Iterable[KvBlockEvent], stop: Optional[threading.Event] = None) -> None:
        for ev in events:
            if stop is not None and stop.is_set():
                break
            if ev is None:
                break
            self.handle(ev)
