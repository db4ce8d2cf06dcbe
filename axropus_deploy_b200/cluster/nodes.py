"""Nodes of the cluster: registries, the snapshot index and node-to-node KV snapshot
transfer.

* :class:`NodeRegistry` -- one row per node (host, router port, GPUs, in-flight jobs,
  HIT / MISS queue depths, capabilities) refreshed by heartbeats; nodes whose last
  heartbeat is older than the TTL (30 s) are left out of :meth:`NodeRegistry.list_nodes`.
* :class:`WorkerRegistry` -- one row per worker (one GPU engine): node, GPU index,
  backend, status, heartbeat.
* :class:`SnapshotIndex` -- where the KV snapshot of a fingerprint lives (ledger
  ``snapshot_locations``), each location tagged with its storage tier (``vram``,
  ``ram``, ``nvme``, from the ``KORITH_SNAPSHOT_{VRAM,RAM,NVME}_DIR`` roots) and sorted
  fastest tier first, most recently used first.
* :func:`estimate_transfer_ms`, :func:`should_transfer_snapshot` -- the cost model of
  moving a snapshot between nodes instead of recomputing its prefix.
* :class:`NodeServer` -- the node's HTTP endpoint ``GET /v1/snapshots/fetch?fingerprint=&org_id=``
  (snapshot bytes, metadata in the ``X-Korith-Snapshot-Meta`` header) and ``GET /health``,
  plus a heartbeat thread into the node registry; :func:`fetch_snapshot_bytes` is its
  client.

Reference: platform/cluster/node_registry.py:10-158, platform/runtime/registry.py:11-115,
platform/cluster/snapshot_index.py:17-195, platform/cluster/snapshot_transfer.py:9-57,
platform/runtime/node_router.py:20-174.
"""
from __future__ import annotations

import json
import logging
import os
import sqlite3
import threading
import time
import urllib.parse
import urllib.request
from datetime import datetime
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional, Tuple

log = logging.getLogger(__name__)

NODE_TTL_S = 30.0
TIERS = ("vram", "ram", "nvme")


class _Db:
    def __init__(self, path: str, schema: str):
        self._mu = threading.Lock()
        self._c = sqlite3.connect(path, check_same_thread=False, timeout=10.0)
        if path != ":memory:":
            self._c.execute("PRAGMA journal_mode=WAL")
        self._c.execute(schema)
        self._c.commit()

    def exec(self, sql: str, args: tuple = ()) -> sqlite3.Cursor:
        with self._mu:
            cur = self._c.execute(sql, args)
            self._c.commit()
            return cur

    def rows(self, sql: str, args: tuple = ()) -> List[Dict[str, Any]]:
        with self._mu:
            cur = self._c.execute(sql, args)
            cols = [d[0] for d in cur.description]
            return [dict(zip(cols, r)) for r in cur.fetchall()]


def _redis(url: str):
    """A Redis client for the optional shared mirror, or None (no URL, or the server does not answer)."""
    if not url:
        return None
    from .netqueues import RespClient

    try:
        c = RespClient(url, timeout_s=2.0)
        c.call("PING")
        return c
    except Exception as e:  # the SQLite copy still serves this node
        log.warning("redis mirror %s unavailable: %s", url, e)
        return None


class NodeRegistry:
    """Nodes and their last heartbeat. With ``redis_url`` every heartbeat is also written to
    Redis (``<prefix>:<node>`` with a TTL of ``ttl_s``, ids in ``<prefix>:ids``), so nodes that
    share no SQLite file see each other; reads prefer Redis and fall back to SQLite."""

    def __init__(self, path: str = ":memory:", ttl_s: float = NODE_TTL_S, redis_url: str = "",
                 key_prefix: str = "korith:nodes"):
        self.ttl_s = ttl_s
        self.redis, self.prefix = _redis(redis_url), key_prefix
        self.db = _Db(path, "CREATE TABLE IF NOT EXISTS nodes (node_id TEXT PRIMARY KEY, host TEXT NOT NULL, "
                            "router_port INTEGER NOT NULL, gpu_count INTEGER NOT NULL, inflight INTEGER NOT NULL, "
                            "queue_depth_hit INTEGER NOT NULL, queue_depth_miss INTEGER NOT NULL, "
                            "capabilities_json TEXT NOT NULL, last_heartbeat REAL NOT NULL)")

    def register_or_heartbeat(self, node_id: str, host: str, router_port: int, gpu_count: int, inflight: int = 0,
                              queue_depth_hit: int = 0, queue_depth_miss: int = 0,
                              capabilities: Optional[Dict[str, Any]] = None, now: Optional[float] = None) -> None:
        t = time.time() if now is None else now
        self.db.exec("INSERT OR REPLACE INTO nodes VALUES (?,?,?,?,?,?,?,?,?)",
                     (node_id, host, int(router_port), int(gpu_count), int(inflight), int(queue_depth_hit),
                      int(queue_depth_miss), json.dumps(capabilities or {}), t))
        if self.redis is not None:
            row = {"node_id": node_id, "host": host, "router_port": int(router_port), "gpu_count": int(gpu_count),
                   "inflight": int(inflight), "queue_depth_hit": int(queue_depth_hit),
                   "queue_depth_miss": int(queue_depth_miss), "capabilities": capabilities or {}, "last_heartbeat": t}
            try:
                self.redis.call("SET", f"{self.prefix}:{node_id}", json.dumps(row), "EX", max(1, int(self.ttl_s)))
                self.redis.call("SADD", f"{self.prefix}:ids", node_id)
            except Exception as e:
                log.warning("redis heartbeat of %s failed: %s", node_id, e)

    def _redis_nodes(self) -> Optional[List[Dict[str, Any]]]:
        if self.redis is None:
            return None
        try:
            out = []
            for nid in self.redis.call("SMEMBERS", f"{self.prefix}:ids") or []:
                v = self.redis.call("GET", f"{self.prefix}:{nid.decode()}")
                if v is not None:
                    out.append(json.loads(v))
            return sorted(out, key=lambda r: r["node_id"])
        except Exception as e:
            log.warning("redis node list failed, using SQLite: %s", e)
            return None

    def _decode(self, r: Dict[str, Any]) -> Dict[str, Any]:
        r = dict(r)
        r["capabilities"] = json.loads(r.pop("capabilities_json") or "{}")
        return r

    def list_nodes(self, healthy_only: bool = True, now: Optional[float] = None) -> List[Dict[str, Any]]:
        t = time.time() if now is None else now
        shared = self._redis_nodes()
        rows = shared if shared is not None else [self._decode(r) for r in self.db.rows("SELECT * FROM nodes ORDER BY node_id")]
        return [r for r in rows if not healthy_only or t - r["last_heartbeat"] <= self.ttl_s]

    def get_node(self, node_id: str) -> Optional[Dict[str, Any]]:
        for r in self._redis_nodes() or []:
            if r["node_id"] == node_id:
                return r
        rows = self.db.rows("SELECT * FROM nodes WHERE node_id=?", (node_id,))
        return self._decode(rows[0]) if rows else None


class WorkerRegistry:
    def __init__(self, path: str = ":memory:"):
        self.db = _Db(path, "CREATE TABLE IF NOT EXISTS workers (worker_id TEXT PRIMARY KEY, node_id TEXT NOT NULL, "
                            "gpu_index INTEGER NOT NULL, backend_id TEXT NOT NULL, status TEXT NOT NULL, "
                            "meta_json TEXT NOT NULL, last_heartbeat REAL NOT NULL)")

    def register(self, worker_id: str, node_id: str, gpu_index: int, backend_id: str, status: str = "idle",
                 meta: Optional[Dict[str, Any]] = None, now: Optional[float] = None) -> None:
        self.db.exec("INSERT OR REPLACE INTO workers VALUES (?,?,?,?,?,?,?)",
                     (worker_id, node_id, int(gpu_index), backend_id, status, json.dumps(meta or {}),
                      time.time() if now is None else now))

    def heartbeat(self, worker_id: str, status: str, meta: Optional[Dict[str, Any]] = None,
                  now: Optional[float] = None) -> bool:
        return self.db.exec("UPDATE workers SET status=?, meta_json=?, last_heartbeat=? WHERE worker_id=?",
                            (status, json.dumps(meta or {}), time.time() if now is None else now,
                             worker_id)).rowcount == 1

    def list_workers(self, max_stale_s: Optional[float] = None, now: Optional[float] = None) -> List[Dict[str, Any]]:
        t = time.time() if now is None else now
        out = []
        for r in self.db.rows("SELECT * FROM workers ORDER BY worker_id"):
            if max_stale_s is not None and t - r["last_heartbeat"] > max_stale_s:
                continue
            r["meta"] = json.loads(r.pop("meta_json") or "{}")
            out.append(r)
        return out


def _iso_ts(s: str) -> float:
    try:
        return datetime.fromisoformat(str(s).replace("Z", "+00:00")).timestamp()
    except ValueError:
        return 0.0


class SnapshotIndex:
    """Snapshot locations over a ledger's ``snapshot_locations`` table. With ``redis_url``
    each (org, fingerprint) also has a Redis hash ``<prefix>:<org>:<fingerprint>`` of its
    locations (field ``<node>:<snapshot>``), read first so that nodes with separate ledgers
    find each other's snapshots; the ledger stays the durable copy."""

    def __init__(self, ledger, tier_roots: Optional[Dict[str, str]] = None, redis_url: str = "",
                 key_prefix: str = "korith:snapshots"):
        self.ledger = ledger
        self._roots = tier_roots
        self.redis, self.prefix = _redis(redis_url), key_prefix

    def _rkey(self, org_id: str, fingerprint_hash: str) -> str:
        return f"{self.prefix}:{org_id}:{fingerprint_hash}"

    def _mirror(self, fingerprint_hash: str, org_id: str) -> None:
        if self.redis is None:
            return
        try:
            args = []
            for r in self.ledger.list_snapshot_locations(fingerprint_hash, org_id):
                args += [f"{r['node_id']}:{r['snapshot_id']}", json.dumps(r, default=str)]
            key = self._rkey(org_id, fingerprint_hash)
            self.redis.call("DEL", key)  # rebuilt whole: locations the ledger pruned disappear too
            if args:
                self.redis.call("HSET", key, *args)
        except Exception as e:
            log.warning("redis snapshot mirror failed: %s", e)

    def tier_roots(self) -> Dict[str, Path]:
        if self._roots is not None:
            return {k: Path(v).resolve() for k, v in self._roots.items() if v}
        out = {}
        for t in TIERS:
            v = os.environ.get(f"KORITH_SNAPSHOT_{t.upper()}_DIR", "").strip()
            if v:
                out[t] = Path(v).expanduser().resolve()
        return out

    def detect_tier(self, snapshot_path: str) -> str:
        if not snapshot_path:
            return "unknown"
        p = Path(snapshot_path).expanduser().resolve()
        for t, root in self.tier_roots().items():
            if p == root or root in p.parents:
                return t
        low = str(snapshot_path).lower()
        for t in TIERS:
            if f"/{t}/" in low:
                return t
        return "unknown"

    def upsert_location(self, fingerprint_hash: str, snapshot_id: str, org_id: str, node_id: str,
                        worker_id: Optional[str], snapshot_path: str, size_bytes: int) -> None:
        from .observability import utc_now

        now = utc_now()
        self.ledger.upsert_snapshot_location(fingerprint_hash, snapshot_id, org_id, node_id, worker_id,
                                             snapshot_path, size_bytes, now, now)
        self._mirror(fingerprint_hash, org_id)

    def _shared_rows(self, fingerprint_hash: str, org_id: str) -> Optional[List[Dict[str, Any]]]:
        if self.redis is None:
            return None
        try:
            flat = self.redis.call("HGETALL", self._rkey(org_id, fingerprint_hash)) or []
            return [json.loads(flat[i + 1]) for i in range(0, len(flat), 2)] or None
        except Exception as e:
            log.warning("redis snapshot lookup failed, using the ledger: %s", e)
            return None

    def get_locations(self, fingerprint_hash: str, org_id: str) -> List[Dict[str, Any]]:
        rows = []
        shared = self._shared_rows(fingerprint_hash, org_id)
        for r in shared if shared is not None else self.ledger.list_snapshot_locations(fingerprint_hash, org_id):
            r = dict(r, storage_tier=self.detect_tier(r["snapshot_path"]))
            rows.append(r)
        rank = {t: i for i, t in enumerate(TIERS)}
        return sorted(rows, key=lambda r: (rank.get(r["storage_tier"], len(TIERS)), -_iso_ts(r["last_used_at"])))

    def mark_used(self, fingerprint_hash: str, org_id: str, node_id: str, snapshot_id: str) -> None:
        from .observability import utc_now

        self.ledger.mark_snapshot_location_used(fingerprint_hash, org_id, node_id, snapshot_id, utc_now())
        self._mirror(fingerprint_hash, org_id)

    def prune_old(self, max_entries_per_fingerprint: int = 8) -> int:
        return self.ledger.prune_snapshot_locations(max_entries_per_fingerprint)


# ---------------------------------------------------------------------- transfer cost model
TIER_READ_GBPS = {"vram": 40.0, "ram": 20.0, "nvme": 6.0, "unknown": 3.0}


def estimate_transfer_ms(size_bytes: int, link_gbps: float, rtt_ms: float, tier: str = "unknown") -> float:
    """Time to move a snapshot: the slower of the source tier's read rate and the link,
    plus one round trip. Rates in GB/s."""
    bw = max(1e-3, min(float(link_gbps), TIER_READ_GBPS.get(tier, TIER_READ_GBPS["unknown"])))
    return max(0, size_bytes) / (bw * 1e9) * 1e3 + max(0.0, rtt_ms)


def should_transfer_snapshot(predicted_lane: str, snapshot_remote: bool, transfer_ms: float,
                             baseline_prefix_ms: float, threshold: float = 0.8) -> bool:
    """Move the snapshot only for a HIT whose snapshot is on another node, when moving
    it costs less than ``threshold`` x recomputing the prefix."""
    if not str(predicted_lane).upper().endswith("HIT") or not snapshot_remote or baseline_prefix_ms <= 0:
        return False
    return transfer_ms < baseline_prefix_ms * threshold


def fetch_snapshot_bytes(host: str, port: int, fingerprint_hash: str, org_id: str,
                         timeout_s: float = 10.0) -> Tuple[bytes, Dict[str, Any]]:
    q = urllib.parse.urlencode({"fingerprint": fingerprint_hash, "org_id": org_id})
    with urllib.request.urlopen(f"http://{host}:{int(port)}/v1/snapshots/fetch?{q}", timeout=timeout_s) as r:
        data = r.read()
        meta_raw = r.headers.get("X-Korith-Snapshot-Meta", "")
    try:
        meta = json.loads(meta_raw) if meta_raw else {}
    except ValueError:
        meta = {}
    return data, meta


def store_snapshot_bytes(path: Path, data: bytes, tok_bytes: Optional[bytes] = None) -> int:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_bytes(data)
    if tok_bytes is not None:
        Path(str(path) + ".tok").write_bytes(tok_bytes)
    return len(data)


class NodeServer:
    """HTTP endpoint of one node; serves the snapshots this node holds."""

    def __init__(self, node_id: str, index: SnapshotIndex, host: str = "127.0.0.1", port: int = 0,
                 registry: Optional[NodeRegistry] = None, status: Optional[Callable[[], Dict[str, Any]]] = None,
                 heartbeat_s: float = 5.0):
        self.node_id = node_id
        self.index = index
        self.registry = registry
        self.status = status or (lambda: {})
        self.heartbeat_s = heartbeat_s
        node = self

        class H(BaseHTTPRequestHandler):
            def log_message(self, *a):
                pass

            def _json(self, code, obj):
                b = json.dumps(obj).encode()
                self.send_response(code)
                self.send_header("Content-Type", "application/json")
                self.send_header("Content-Length", str(len(b)))
                self.end_headers()
                self.wfile.write(b)

            def do_GET(self):
                u = urllib.parse.urlparse(self.path)
                q = urllib.parse.parse_qs(u.query)
                if u.path == "/health":
                    return self._json(200, {"status": "ok", "node_id": node.node_id})
                if u.path != "/v1/snapshots/fetch":
                    return self._json(404, {"error": "not found"})
                fp, org = q.get("fingerprint", [""])[0], q.get("org_id", ["default"])[0]
                for loc in node.index.get_locations(fp, org):
                    if loc["node_id"] != node.node_id or not Path(loc["snapshot_path"]).exists():
                        continue
                    data = Path(loc["snapshot_path"]).read_bytes()
                    tok = Path(loc["snapshot_path"] + ".tok")
                    meta = {"fingerprint_hash": fp, "snapshot_id": loc["snapshot_id"], "node_id": node.node_id,
                            "size_bytes": len(data), "storage_tier": loc["storage_tier"],
                            "tokens_hex": tok.read_bytes().hex() if tok.exists() else ""}
                    node.index.mark_used(fp, org, node.node_id, loc["snapshot_id"])
                    self.send_response(200)
                    self.send_header("Content-Type", "application/octet-stream")
                    self.send_header("Content-Length", str(len(data)))
                    self.send_header("X-Korith-Snapshot-Meta", json.dumps(meta))
                    self.end_headers()
                    self.wfile.write(data)
                    return
                return self._json(404, {"error": "snapshot not on this node"})

        self.httpd = ThreadingHTTPServer((host, port), H)
        self.host, self.port = self.httpd.server_address[0], self.httpd.server_address[1]
        self._stop = threading.Event()
        self._threads: List[threading.Thread] = []

    def heartbeat_once(self) -> None:
        if self.registry is None:
            return
        st = self.status()
        self.registry.register_or_heartbeat(self.node_id, self.host, self.port, int(st.get("gpu_count", 1)),
                                            int(st.get("inflight", 0)), int(st.get("queue_depth_hit", 0)),
                                            int(st.get("queue_depth_miss", 0)), st.get("capabilities", {}))

    def start(self) -> "NodeServer":
        t = threading.Thread(target=self.httpd.serve_forever, daemon=True)
        t.start()
        self._threads.append(t)

        def beat():
            while not self._stop.is_set():
                try:
                    self.heartbeat_once()
                except Exception:  # a registry outage must not stop the node
                    pass
                self._stop.wait(self.heartbeat_s)

        hb = threading.Thread(target=beat, daemon=True)
        hb.start()
        self._threads.append(hb)
        return self

    def stop(self) -> None:
        self._stop.set()
        self.httpd.shutdown()
        self.httpd.server_close()
