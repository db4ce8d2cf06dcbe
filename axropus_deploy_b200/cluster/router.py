"""Cluster router: picks the worker (one GPU engine on some node) for a request.

``submit`` canonicalises the prompt, derives the AMF lookup hash (FNV-1a64 of
``tenant:prompt``, the reference's ``amf_lookup_hash``) and the pool key of the token
prefix, checks the context budget, predicts the lane and chooses a route:

* ``amf_local`` -- a live worker already holds the prefix (coordinator lookup): send the
  request there, restore instead of prefill;
* ``amf_transfer`` -- the prefix lives on another node than the least-loaded worker's:
  move the KV if ``bytes / link_gbps`` beats recomputing (``tokens / prefill_tok_s``),
  else recompute there;
* ``cold`` -- nobody holds it: least-loaded worker, prefill.

Lanes: ``SPEC_HIT`` / ``HIT`` (prefix held; SPEC_ when the worker runs speculative
decoding), ``SPEC_MISS`` / ``MISS``. The chosen worker's queue receives the job.

Reference: platform/runtime/cluster_router.py:108-316 (submit: validate, canonicalise,
hashes, preflight, lane, route, enqueue) and :408 (``_select_route``).
"""
from __future__ import annotations

import re
import unicodedata
from dataclasses import dataclass, field
from typing import Dict, List, Optional

from ..amf.keys import FNV_OFFSET, fnv1a_bytes, pool_key


@dataclass
class WorkerInfo:
    worker_id: str
    node_id: str
    load: float = 0.0               # queued + running tokens (or any load measure)
    max_ctx: int = 32768
    spec: bool = False
    prefill_tok_s: float = 40000.0  # cold prefill rate of this worker's model
    kv_bytes_per_token: int = 131072
    queue: object = None            # anything with enqueue(item)


@dataclass
class Route:
    worker: WorkerInfo
    kind: str                       # amf_local | amf_transfer | recompute | cold
    lane: str
    amf_lookup_hash: int
    prefix_key: str
    source_node: Optional[str] = None
    est_ms: float = 0.0
    reasons: List[str] = field(default_factory=list)


def canonicalize(prompt: str, collapse_whitespace: bool = True, nfc: bool = True) -> str:
    s = unicodedata.normalize("NFC", prompt) if nfc else prompt
    if collapse_whitespace:
        s = re.sub(r"[ \t]+", " ", s)
        s = re.sub(r"\n{3,}", "\n\n", s)
    return s.strip()


def amf_lookup_hash(tenant_id: str, prompt: str) -> int:
    return fnv1a_bytes(f"{tenant_id}:{prompt}".encode("utf-8"), FNV_OFFSET)


class ClusterRouter:
    def __init__(self, workers: List[WorkerInfo], coordinator=None, link_gbps: float = 50.0,
                 prefix_tokens: int = 4096):
        self.workers: Dict[str, WorkerInfo] = {w.worker_id: w for w in workers}
        self.coord = coordinator          # CoordinatorClient or AmfCoordinator (lookup(prefix, tenant))
        self.link_gbps = link_gbps        # inter-node bandwidth for a KV transfer
        self.prefix_tokens = prefix_tokens
        self.stat: Dict[str, int] = {}

    def _locations(self, key: str, tenant: str) -> List[dict]:
        if self.coord is None:
            return []
        try:
            if hasattr(self.coord, "base"):  # HTTP client
                return self.coord.lookup(key, tenant)
            return self.coord.lookup(tenant, key)
        except Exception:  # fail open
            return []

    def submit(self, prompt: str, tenant_id: str = "default", max_tokens: int = 256, job: Optional[dict] = None,
               tokens: Optional[List[int]] = None) -> Route:
        if not self.workers:
            raise RuntimeError("no workers registered")
        text = canonicalize(prompt)
        toks = tokens if tokens is not None else list(text.encode("utf-8"))  # byte tokenizer fallback
        n = len(toks)
        fits = [w for w in self.workers.values() if n + max_tokens <= w.max_ctx]
        if not fits:
            raise ValueError(f"prompt of {n} tokens + {max_tokens} exceeds every worker's context")
        pre = toks[: min(n, self.prefix_tokens) // 16 * 16]
        key = pool_key(pre) if pre else ""
        lh = amf_lookup_hash(tenant_id, text)
        least = min(fits, key=lambda w: w.load)
        holders = [self.workers[l["worker_id"]] for l in self._locations(key, tenant_id)
                   if l.get("worker_id") in self.workers and self.workers[l["worker_id"]] in fits] if key else []
        reasons: List[str] = []
        if holders:
            best = min(holders, key=lambda w: w.load)
            # the holder wins unless its extra load (tokens) exceeds the prefill it saves
            if best is least or best.load - least.load <= len(pre):
                kind, worker, src, est = "amf_local", best, best.node_id, 0.0
                reasons.append("prefix held by a live worker")
            else:
                transfer_ms = len(pre) * least.kv_bytes_per_token / (self.link_gbps * 1e9) * 1e3
                recompute_ms = len(pre) / least.prefill_tok_s * 1e3
                if best.node_id == least.node_id or transfer_ms < recompute_ms:
                    kind, worker, src, est = "amf_transfer", least, best.node_id, transfer_ms
                    reasons.append(f"holder busy; transfer {transfer_ms:.1f} ms < recompute {recompute_ms:.1f} ms")
                else:
                    kind, worker, src, est = "recompute", least, None, recompute_ms
                    reasons.append(f"holder busy; recompute {recompute_ms:.1f} ms <= transfer {transfer_ms:.1f} ms")
        else:
            kind, worker, src, est = "cold", least, None, len(pre) / least.prefill_tok_s * 1e3
            reasons.append("prefix not held")
        hit = kind in ("amf_local", "amf_transfer")
        lane = ("SPEC_" if worker.spec else "") + ("HIT" if hit else "MISS")
        route = Route(worker, kind, lane, lh, key, src, est, reasons)
        worker.load += n + max_tokens
        self.stat[kind] = self.stat.get(kind, 0) + 1
        if worker.queue is not None:
            worker.queue.enqueue(dict(job or {}, prompt=text, tenant_id=tenant_id, max_tokens=max_tokens, route=kind,
                                      lane=lane, amf_lookup_hash=lh, prefix_key=key, source_node=src))
        return route
