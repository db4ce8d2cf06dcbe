"""AMF coordinator: which node / worker holds which prefix, across the cluster.

Inside one node the sharded G1 pool already answers this (the shard directory in shared
memory); across nodes a small service keeps the index. Records are keyed by
``tenant:prefix_hash`` and list every node holding the prefix, with the worker and free-form
metadata (tier, tokens, format). They persist in SQLite (WAL) so a restarted coordinator
keeps its index. Nodes report liveness with heartbeats (optionally carrying their full
entry list, which replaces what the node had registered); lookups skip nodes whose last
heartbeat is older than ``node_ttl_s``.

HTTP (stdlib server, JSON bodies): ``GET /health``, ``GET /stats``, ``GET /metrics``
(Prometheus text), ``GET /lookup?tenant_id=&prefix_hash=``, ``POST /register``,
``POST /heartbeat``, ``DELETE /evict?tenant_id=&prefix_hash=[&node_id=]``.
:class:`CoordinatorClient` uses short timeouts and fails open: any error reads as "no
location known", so a dead coordinator only costs cache locality, never a request.

Reference: platform/runtime/amf_coordinator.py:18-329 (SQLite index, the same endpoint
names) and platform/runtime/amf_coordinator_client.py:49-139 (0.25 s timeout, fail-open).
"""
from __future__ import annotations

import json
import sqlite3
import threading
import time
import urllib.error
import urllib.parse
import urllib.request
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Any, Dict, List, Optional, Tuple


def _clean(s: Any, keep: str = "-_.", default: str = "") -> str:
    t = "".join(c for c in str(s or "").strip() if c.isalnum() or c in keep)[:128]
    return t or default


def composite_key(tenant_id: str, prefix_hash: str) -> str:
    return f"{_clean(tenant_id, default='default')}:{_clean(prefix_hash, keep='').lower()}"


class AmfCoordinator:
    SCHEMA = """
    CREATE TABLE IF NOT EXISTS locations (
        key TEXT NOT NULL, node TEXT NOT NULL, worker TEXT NOT NULL DEFAULT '',
        meta TEXT NOT NULL DEFAULT '{}', updated REAL NOT NULL, PRIMARY KEY (key, node));
    CREATE INDEX IF NOT EXISTS loc_node ON locations (node);
    CREATE TABLE IF NOT EXISTS nodes (node TEXT PRIMARY KEY, seen REAL NOT NULL);
    """

    def __init__(self, db_path: str = ":memory:", node_ttl_s: float = 30.0):
        self.node_ttl_s = node_ttl_s
        self._mu = threading.Lock()
        self._db = sqlite3.connect(db_path, check_same_thread=False)
        if db_path != ":memory:":
            self._db.execute("PRAGMA journal_mode=WAL")
        self._db.executescript(self.SCHEMA)
        self._db.commit()
        self.stat = {"lookups": 0, "hits": 0, "registers": 0, "heartbeats": 0, "evictions": 0}

    # ------------------------------------------------------------------ index
    def register(self, tenant_id: str, prefix_hash: str, node_id: str, worker_id: str = "",
                 metadata: Optional[dict] = None, now: Optional[float] = None) -> bool:
        node = _clean(node_id)
        if not node or not _clean(prefix_hash, keep=""):
            return False
        t = time.time() if now is None else now
        with self._mu:
            self._db.execute("INSERT OR REPLACE INTO locations VALUES (?, ?, ?, ?, ?)",
                             (composite_key(tenant_id, prefix_hash), node, _clean(worker_id),
                              json.dumps(metadata or {}), t))
            self._db.execute("INSERT OR REPLACE INTO nodes VALUES (?, ?)", (node, t))
            self._db.commit()
            self.stat["registers"] += 1
        return True

    def heartbeat(self, node_id: str, entries: Optional[List[dict]] = None, now: Optional[float] = None) -> bool:
        """Mark the node alive; with ``entries`` (tenant_id, prefix_hash, worker_id,
        metadata) the node's registrations are replaced by exactly that list."""
        node = _clean(node_id)
        if not node:
            return False
        t = time.time() if now is None else now
        with self._mu:
            self._db.execute("INSERT OR REPLACE INTO nodes VALUES (?, ?)", (node, t))
            if entries is not None:
                self._db.execute("DELETE FROM locations WHERE node = ?", (node,))
                self._db.executemany("INSERT OR REPLACE INTO locations VALUES (?, ?, ?, ?, ?)", [
                    (composite_key(e.get("tenant_id", "default"), e.get("prefix_hash", "")), node,
                     _clean(e.get("worker_id", "")), json.dumps(e.get("metadata", {})), t)
                    for e in entries if _clean(e.get("prefix_hash", ""), keep="")])
            self._db.commit()
            self.stat["heartbeats"] += 1
        return True

    def lookup(self, tenant_id: str, prefix_hash: str, now: Optional[float] = None) -> List[dict]:
        t = time.time() if now is None else now
        with self._mu:
            rows = self._db.execute(
                "SELECT l.node, l.worker, l.meta, l.updated FROM locations l JOIN nodes n ON n.node = l.node "
                "WHERE l.key = ? AND n.seen >= ? ORDER BY l.updated DESC",
                (composite_key(tenant_id, prefix_hash), t - self.node_ttl_s)).fetchall()
            self.stat["lookups"] += 1
            self.stat["hits"] += 1 if rows else 0
        return [{"node_id": n, "worker_id": w, "metadata": json.loads(m), "updated_at": u} for n, w, m, u in rows]

    def evict(self, tenant_id: str, prefix_hash: str, node_id: Optional[str] = None) -> int:
        with self._mu:
            if node_id:
                cur = self._db.execute("DELETE FROM locations WHERE key = ? AND node = ?",
                                       (composite_key(tenant_id, prefix_hash), _clean(node_id)))
            else:
                cur = self._db.execute("DELETE FROM locations WHERE key = ?", (composite_key(tenant_id, prefix_hash),))
            self._db.commit()
            self.stat["evictions"] += cur.rowcount
            return cur.rowcount

    def stats(self, now: Optional[float] = None) -> Dict[str, Any]:
        t = time.time() if now is None else now
        with self._mu:
            n_loc = self._db.execute("SELECT COUNT(*) FROM locations").fetchone()[0]
            n_keys = self._db.execute("SELECT COUNT(DISTINCT key) FROM locations").fetchone()[0]
            live = self._db.execute("SELECT COUNT(*) FROM nodes WHERE seen >= ?", (t - self.node_ttl_s,)).fetchone()[0]
        return dict(self.stat, locations=n_loc, prefixes=n_keys, live_nodes=live)

    def prometheus(self) -> str:
        s = self.stats()
        return "".join(f"axropus_coordinator_{k} {v}\n" for k, v in s.items())


class _Handler(BaseHTTPRequestHandler):
    coord: AmfCoordinator = None  # set by serve_coordinator

    def log_message(self, fmt, *args):  # quiet
        pass

    def _send(self, code: int, payload: Any, ctype: str = "application/json") -> None:
        body = payload.encode() if isinstance(payload, str) else json.dumps(payload).encode()
        self.send_response(code)
        self.send_header("Content-Type", ctype)
        self.send_header("Content-Length", str(len(body)))
        self.end_headers()
        self.wfile.write(body)

    def _body(self) -> dict:
        n = int(self.headers.get("Content-Length") or 0)
        try:
            return json.loads(self.rfile.read(n) or b"{}")
        except ValueError:
            return {}

    def do_GET(self):
        u = urllib.parse.urlparse(self.path)
        q = dict(urllib.parse.parse_qsl(u.query))
        if u.path == "/health":
            return self._send(200, {"ok": True})
        if u.path == "/stats":
            return self._send(200, self.coord.stats())
        if u.path == "/metrics":
            return self._send(200, self.coord.prometheus(), "text/plain; version=0.0.4")
        if u.path == "/lookup":
            return self._send(200, {"locations": self.coord.lookup(q.get("tenant_id", "default"),
                                                                   q.get("prefix_hash", ""))})
        self._send(404, {"error": "not found"})

    def do_POST(self):
        u = urllib.parse.urlparse(self.path)
        b = self._body()
        if u.path == "/register":
            ok = self.coord.register(b.get("tenant_id", "default"), b.get("prefix_hash", ""), b.get("node_id", ""),
                                     b.get("worker_id", ""), b.get("metadata"))
            return self._send(200 if ok else 400, {"ok": ok})
        if u.path == "/heartbeat":
            ok = self.coord.heartbeat(b.get("node_id", ""), b.get("entries"))
            return self._send(200 if ok else 400, {"ok": ok})
        self._send(404, {"error": "not found"})

    def do_DELETE(self):
        u = urllib.parse.urlparse(self.path)
        q = dict(urllib.parse.parse_qsl(u.query))
        if u.path == "/evict":
            n = self.coord.evict(q.get("tenant_id", "default"), q.get("prefix_hash", ""), q.get("node_id"))
            return self._send(200, {"evicted": n})
        self._send(404, {"error": "not found"})


def serve_coordinator(coord: AmfCoordinator, host: str = "127.0.0.1", port: int = 0) -> Tuple[ThreadingHTTPServer, int]:
    """Start the HTTP server in a daemon thread; returns (server, port)."""
    handler = type("CoordinatorHandler", (_Handler,), {"coord": coord})
    srv = ThreadingHTTPServer((host, port), handler)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv, srv.server_address[1]


class CoordinatorClient:
    """Fail-open client: errors and timeouts read as 'nothing known' / 'not stored'."""

    def __init__(self, base_url: str, timeout_s: float = 0.25):
        self.base = base_url.rstrip("/")
        self.timeout_s = max(0.05, float(timeout_s))
        self.errors = 0

    def _req(self, method: str, path: str, body: Optional[dict] = None) -> Optional[dict]:
        data = json.dumps(body).encode() if body is not None else None
        req = urllib.request.Request(self.base + path, data=data, method=method,
                                     headers={"Content-Type": "application/json"})
        try:
            with urllib.request.urlopen(req, timeout=self.timeout_s) as r:
                return json.loads(r.read() or b"{}")
        except (urllib.error.URLError, OSError, ValueError):
            self.errors += 1
            return None

    def lookup(self, prefix_hash: str, tenant_id: str = "default") -> List[dict]:
        q = urllib.parse.urlencode({"tenant_id": tenant_id, "prefix_hash": prefix_hash})
        r = self._req("GET", f"/lookup?{q}")
        return (r or {}).get("locations", [])

    def register(self, prefix_hash: str, node_id: str, worker_id: str = "", tenant_id: str = "default",
                 metadata: Optional[dict] = None) -> bool:
        r = self._req("POST", "/register", {"tenant_id": tenant_id, "prefix_hash": prefix_hash, "node_id": node_id,
                                            "worker_id": worker_id, "metadata": metadata or {}})
        return bool(r and r.get("ok"))

    def heartbeat(self, node_id: str, entries: Optional[List[dict]] = None) -> bool:
        r = self._req("POST", "/heartbeat", {"node_id": node_id, "entries": entries})
        return bool(r and r.get("ok"))

    def evict(self, prefix_hash: str, tenant_id: str = "default", node_id: Optional[str] = None) -> int:
        q = {"tenant_id": tenant_id, "prefix_hash": prefix_hash}
        if node_id:
            q["node_id"] = node_id
        r = self._req("DELETE", "/evict?" + urllib.parse.urlencode(q))
        return int((r or {}).get("evicted", 0))
