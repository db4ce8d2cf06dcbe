"""HTTP gateway of the control plane (stdlib ``ThreadingHTTPServer``, JSON bodies).

Authentication: ``Authorization: Bearer <api key>``; keys are stored as
sha256(``KORITH_API_KEY_SALT`` + key) in the ledger (the salt must be set, and not to
the placeholder ``korith_default_salt``); revoked keys get 403. Limits, checked before
a job is accepted (429 with ``Retry-After``):

* per tenant: a token bucket of ``KORITH_TENANT_RPS`` requests/s (burst
  ``KORITH_RATE_LIMIT_BURST`` x rate);
* per organisation: the API key's requests/minute and tokens/minute in 60-second
  windows, times the burst factor (:class:`RateLimiter`, SQLite when
  ``KORITH_RATE_LIMIT_DB`` is set so that several gateway processes share the count).

Endpoints: ``GET /health``, ``/ready``, ``/metrics`` (Prometheus text, no auth);
``GET /v1/jobs``, ``/v1/jobs/{id}`` (+ ``/metrics``, ``/events``, ``/logs``),
``/v1/health``, ``/v1/alerts``, ``/v1/workers``, ``/v1/queue_status``,
``/v1/capabilities``, ``/v1/cluster/nodes``, ``/v1/cluster/routing?fingerprint=``,
``/v1/snapshots/locations?fingerprint=``, ``/v1/replay/status?fingerprint=``,
``/v1/spec/status?fingerprint=``, ``/v1/kernels/status``, ``/v1/kpi/summary``,
``/v1/metrics/tenant/{tenant}``; ``POST /v1/jobs``, ``/v1/billing/report``,
``/v1/jobs/{id}/restore``. Every response carries ``X-Request-Id``.

Reference: platform/gateway/http_server.py:29-556 (endpoint set, auth and limit order),
platform/gateway/auth.py (salted key hash, bearer parsing), platform/gateway/rate_limit.py:22-138.
"""
from __future__ import annotations

import hashlib
import json
import os
import sqlite3
import threading
import time
import uuid
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Any, Dict, Optional, Tuple
from urllib.parse import parse_qs, urlparse

from .observability import GLOBAL_METRICS, ArtifactStore, utc_now


class AuthError(Exception):
    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status, self.msg = status, msg


def api_key_salt() -> str:
    s = os.environ.get("KORITH_API_KEY_SALT", "").strip()
    if not s or s == "korith_default_salt":
        raise RuntimeError("KORITH_API_KEY_SALT must be set to a secret value")
    return s


def hash_api_key(raw: str) -> str:
    return hashlib.sha256((api_key_salt() + raw).encode("utf-8")).hexdigest()


def issue_api_key(ledger, key_id: str, org_id: str, rpm: int = 600, tpm: int = 120000,
                  permissions: Optional[Dict[str, Any]] = None) -> str:
    """Create a key (returned once, stored only hashed)."""
    raw = f"kth_{key_id}_{uuid.uuid4().hex}{uuid.uuid4().hex[:8]}"
    ledger.create_api_key(key_id, hash_api_key(raw), org_id, utc_now(), tpm, rpm, json.dumps(permissions or {}))
    return raw


def authenticate(headers, ledger) -> Dict[str, Any]:
    h = headers.get("Authorization") or headers.get("authorization") or ""
    parts = h.split(" ", 1)
    if not h:
        raise AuthError(401, "missing authorization header")
    if len(parts) != 2 or parts[0].lower() != "bearer" or not parts[1].strip():
        raise AuthError(401, "invalid authorization header")
    try:
        rec = ledger.get_api_key_by_hash(hash_api_key(parts[1].strip()))
    except RuntimeError as e:
        raise AuthError(503, f"auth backend unavailable: {e}")
    if rec is None:
        raise AuthError(401, "invalid api key")
    if rec.get("revoked_at"):
        raise AuthError(403, "api key revoked")
    try:
        perms = json.loads(rec.get("permissions_json") or "{}")
    except ValueError:
        perms = {}
    return {"key_id": rec["key_id"], "org_id": rec["org_id"], "permissions": perms,
            "rpm": int(rec["rate_limit_rpm"]), "tpm": int(rec["rate_limit_tpm"])}


# Atomic check-and-consume of one request and its tokens in a 60-second window. KEYS:
# request counter, token counter; ARGV: request cap, token cap, tokens, TTL seconds.
# Returns {1, 0} when consumed, {0, 1} over the request cap, {0, 2} over the token cap;
# a refusal changes nothing. Redis runs a script atomically, so no other gateway can
# interleave between the check and the increments, and the TTL is set in the same step.
RATE_LIMIT_LUA = """
local r = tonumber(redis.call('GET', KEYS[1]) or '0')
local t = tonumber(redis.call('GET', KEYS[2]) or '0')
if r + 1 > tonumber(ARGV[1]) then return {0, 1} end
if t + tonumber(ARGV[3]) > tonumber(ARGV[2]) then return {0, 2} end
redis.call('INCRBY', KEYS[1], 1)
redis.call('EXPIRE', KEYS[1], ARGV[4])
redis.call('INCRBY', KEYS[2], ARGV[3])
redis.call('EXPIRE', KEYS[2], ARGV[4])
return {1, 0}
"""


class RateLimiter:
    """Requests and tokens per organisation in 60-second windows: in memory, in SQLite
    (``KORITH_RATE_LIMIT_DB``), or in Redis (``KORITH_RATE_LIMIT_BACKEND=redis`` with
    ``KORITH_REDIS_URL``), where every gateway of a deployment shares one budget: counters
    ``korith:rl:{req,tok}:<org>:<window>`` are checked and consumed by one atomic script
    (:data:`RATE_LIMIT_LUA`; refusals use no quota). The script is sent at most once per
    request: if the connection drops mid-call the request is decided by this gateway's
    in-memory window instead, so quota is never spent twice."""

    def __init__(self, db_path: Optional[str] = None, burst_factor: Optional[float] = None,
                 redis_url: Optional[str] = None):
        self.burst = max(1.0, float(burst_factor if burst_factor is not None else
                                    os.environ.get("KORITH_RATE_LIMIT_BURST", "2.0") or 2.0))
        self._mu = threading.Lock()
        self._mem: Dict[Tuple[str, int], list] = {}
        if redis_url is None and os.environ.get("KORITH_RATE_LIMIT_BACKEND", "").strip().lower() == "redis":
            redis_url = os.environ.get("KORITH_REDIS_URL", "redis://127.0.0.1:6379/0")
        self._redis = None
        if redis_url:
            from .netqueues import RespClient

            self._redis = RespClient(redis_url)
        path = db_path or os.environ.get("KORITH_RATE_LIMIT_DB", "")
        self._db = sqlite3.connect(path, check_same_thread=False, timeout=5.0) if path else None
        if self._db is not None:
            self._db.execute("CREATE TABLE IF NOT EXISTS rate_limit_windows (org_id TEXT NOT NULL, window_epoch "
                             "INTEGER NOT NULL, request_count INTEGER NOT NULL, token_count INTEGER NOT NULL, "
                             "PRIMARY KEY(org_id, window_epoch))")
            self._db.commit()

    def check_and_consume(self, org_id: str, tokens: int, rpm: int, tpm: int,
                          now: Optional[float] = None) -> Dict[str, Any]:
        t = int(time.time() if now is None else now)
        win = t - t % 60
        rcap, tcap = max(1, int(rpm * self.burst)), max(1, int(tpm * self.burst))
        if self._redis is not None:
            rk, tk = f"korith:rl:req:{org_id}:{win}", f"korith:rl:tok:{org_id}:{win}"
            try:
                ok, why = self._redis.call("EVAL", RATE_LIMIT_LUA, 2, rk, tk, rcap, tcap, int(tokens), 180,
                                           retry=False)
            except (ConnectionError, OSError):
                ok = None  # Redis unreachable: this gateway's own window decides
            if ok is not None:
                if int(ok):
                    return {"allowed": True, "reason": "ok"}
                return {"allowed": False, "reason": "rpm_exceeded" if int(why) == 1 else "tpm_exceeded",
                        "retry_after": 60 - t % 60}
        with self._mu:
            if self._db is not None:
                self._db.execute("DELETE FROM rate_limit_windows WHERE window_epoch < ?", (win - 120,))
                row = self._db.execute("SELECT request_count, token_count FROM rate_limit_windows WHERE org_id=? "
                                       "AND window_epoch=?", (org_id, win)).fetchone()
                reqs, toks = row if row else (0, 0)
            else:
                for k in [k for k in self._mem if k[1] < win - 120]:
                    del self._mem[k]
                reqs, toks = self._mem.get((org_id, win), [0, 0])
            if reqs + 1 > rcap:
                return {"allowed": False, "reason": "rpm_exceeded", "retry_after": 60 - t % 60}
            if toks + tokens > tcap:
                return {"allowed": False, "reason": "tpm_exceeded", "retry_after": 60 - t % 60}
            if self._db is not None:
                self._db.execute("INSERT INTO rate_limit_windows VALUES (?,?,1,?) ON CONFLICT(org_id, window_epoch) "
                                 "DO UPDATE SET request_count=request_count+1, token_count=token_count+?",
                                 (org_id, win, tokens, tokens))
                self._db.commit()
            else:
                self._mem[(org_id, win)] = [reqs + 1, toks + tokens]
        return {"allowed": True, "reason": "ok"}


class TokenBucket:
    def __init__(self, rate: float, burst: float):
        self.rate, self.cap = rate, max(1.0, burst)
        self._b: Dict[str, Tuple[float, float]] = {}
        self._mu = threading.Lock()

    def take(self, key: str, now: Optional[float] = None) -> float:
        """0 when admitted, else the seconds until a token is available."""
        t = time.monotonic() if now is None else now
        with self._mu:
            level, last = self._b.get(key, (self.cap, t))
            level = min(self.cap, level + (t - last) * self.rate)
            if level >= 1.0:
                self._b[key] = (level - 1.0, t)
                return 0.0
            self._b[key] = (level, t)
            return (1.0 - level) / self.rate


def active_alerts(plane, metrics=GLOBAL_METRICS) -> list:
    snap = metrics.snapshot()
    c = snap["counters"]
    ok = sum(v for k, v in c.items() if k.startswith("korith_jobs_total") and 'status="ok"' in k)
    bad = sum(v for k, v in c.items() if k.startswith("korith_jobs_total") and 'status="failed"' in k)
    out = []
    rate = float(os.environ.get("KORITH_ALERT_FAILURE_RATE", "0.05"))
    if ok + bad > 0 and bad / (ok + bad) > rate:
        out.append({"name": "job_failure_rate", "severity": "warning", "value": bad / (ok + bad)})
    depth_max = float(os.environ.get("KORITH_ALERT_QUEUE_DEPTH", "256"))
    for w in plane.queue_status():
        d = sum(w["depths"].values())
        if d > depth_max:
            out.append({"name": "queue_depth", "severity": "critical", "worker": w["worker_id"], "value": d})
    for g in plane.ledger.list_replay_governance(1000):
        if g["replay_disabled"] and g["corruption_detected"]:
            out.append({"name": "snapshot_corruption", "severity": "warning", "fingerprint": g["fingerprint_hash"]})
    return out


def make_handler(plane, limiter: RateLimiter, tenant_bucket: TokenBucket):
    class Handler(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"

        def log_message(self, *a):
            pass

        def _send(self, code: int, obj: Any, rid: str, headers: Optional[Dict[str, str]] = None,
                  ctype: str = "application/json") -> None:
            b = obj if isinstance(obj, bytes) else json.dumps(obj, default=str).encode()
            self.send_response(code)
            self.send_header("Content-Type", ctype)
            self.send_header("Content-Length", str(len(b)))
            self.send_header("X-Request-Id", rid)
            for k, v in (headers or {}).items():
                self.send_header(k, v)
            self.end_headers()
            self.wfile.write(b)

        def _rid(self) -> str:
            return self.headers.get("X-Request-Id") or uuid.uuid4().hex

        def _body(self) -> Any:
            n = int(self.headers.get("Content-Length", "0") or 0)
            raw = self.rfile.read(n).decode("utf-8", "replace") if n > 0 else ""
            return json.loads(raw) if raw.strip() else {}

        def _auth(self, rid: str) -> Optional[Dict[str, Any]]:
            try:
                return authenticate(self.headers, plane.ledger)
            except AuthError as e:
                self._send(e.status, {"error": e.msg}, rid)
                return None

        def do_GET(self):
            rid = self._rid()
            u = urlparse(self.path)
            p, q = u.path, parse_qs(u.query)
            if p == "/health":
                return self._send(200, {"status": "ok"}, rid)
            if p == "/ready":
                ready = bool(plane.get_workers())
                return self._send(200 if ready else 503, {"ready": ready}, rid)
            if p == "/metrics":
                reg = getattr(plane, "metrics", GLOBAL_METRICS)
                return self._send(200, reg.render_prometheus().encode(), rid,
                                  ctype="text/plain; version=0.0.4")
            if not p.startswith("/v1/"):
                return self._send(404, {"error": "not found"}, rid)
            auth = self._auth(rid)
            if auth is None:
                return
            org = auth["org_id"]
            fp = q.get("fingerprint", [""])[0]
            need_fp = {"/v1/cluster/routing", "/v1/snapshots/locations", "/v1/replay/status", "/v1/spec/status"}
            if p in need_fp and not fp:
                return self._send(400, {"error": "fingerprint query param required"}, rid)
            simple = {
                "/v1/health": lambda: {"status": "ok"},
                "/v1/alerts": lambda: {"alerts": active_alerts(plane, getattr(plane, "metrics", GLOBAL_METRICS))},
                "/v1/workers": lambda: {"workers": plane.get_workers()},
                "/v1/queue_status": lambda: {"queue": plane.queue_status()},
                "/v1/capabilities": lambda: {"capabilities": plane.capabilities()},
                "/v1/cluster/nodes": lambda: {"nodes": plane.cluster_nodes()},
                "/v1/cluster/routing": lambda: plane.routing_debug(fp, org),
                "/v1/snapshots/locations": lambda: plane.snapshot_locations(fp, org),
                "/v1/replay/status": lambda: plane.replay_status(fp),
                "/v1/spec/status": lambda: plane.spec_status(fp, org),
                "/v1/kernels/status": lambda: plane.kernels_status(),
            }
            if p in simple:
                return self._send(200, simple[p](), rid)
            if p == "/v1/jobs":
                try:
                    limit = int(q.get("limit", ["20"])[0])
                except ValueError:
                    limit = 20
                return self._send(200, {"jobs": plane.list_jobs(limit, org_id=org)}, rid)
            if p == "/v1/kpi/summary":
                try:
                    limit = max(1, int(q.get("limit", ["500"])[0]))
                    cost = float(q.get("gpu_hourly_cost", ["2.5"])[0])
                except ValueError:
                    limit, cost = 500, 2.5
                return self._send(200, plane.kpi_summary(org, limit, cost), rid)
            if p.startswith("/v1/metrics/tenant/"):
                tenant = p.split("/")[4] if len(p.split("/")) > 4 else ""
                if not tenant:
                    return self._send(400, {"error": "tenant_id required"}, rid)
                return self._send(200, plane.tenant_metrics(tenant, org), rid)
            if p.startswith("/v1/jobs/"):
                parts = p.split("/")
                rec = plane.get_job(parts[3] if len(parts) > 3 else "", org_id=org)
                if rec is None:
                    return self._send(404, {"error": "job not found"}, rid)
                if p.endswith("/metrics"):
                    mp = rec.get("metrics_path")
                    return self._send(200, json.loads(open(mp).read()) if mp and os.path.exists(mp)
                                      else {"metrics_path": mp}, rid)
                if p.endswith("/events"):
                    ep = rec.get("events_path")
                    return self._send(200, {"events": ArtifactStore.read_events(ep)} if ep else {"events": []}, rid)
                if p.endswith("/logs"):
                    lp = rec.get("log_path")
                    return self._send(200, {"log": open(lp).read() if lp and os.path.exists(lp) else ""}, rid)
                return self._send(200, rec, rid)
            return self._send(404, {"error": "not found"}, rid)

        def do_POST(self):
            rid = self._rid()
            p = urlparse(self.path).path
            if not p.startswith("/v1/"):
                return self._send(404, {"error": "not found"}, rid)
            auth = self._auth(rid)
            if auth is None:
                return
            org = auth["org_id"]
            try:
                body = self._body()
            except ValueError as e:
                return self._send(400, {"error": f"invalid json body: {e}", "code": "INVALID_JSON"}, rid)
            if p == "/v1/jobs":
                if not isinstance(body, dict):
                    return self._send(400, {"error": "jobspec must be an object", "code": "INVALID_JOBSPEC"}, rid)
                tenant = str(body.get("tenant_id") or auth["permissions"].get("tenant_id") or org)
                wait = tenant_bucket.take(tenant)
                if wait > 0:
                    return self._send(429, {"error": "tenant rate limit", "tenant_id": tenant,
                                            "retry_after": wait}, rid, {"Retry-After": str(max(1, int(wait + 0.999)))})
                est = len(str(body.get("prompt", ""))) + int(body.get("max_tokens", 64) or 0)
                d = limiter.check_and_consume(org, est, auth["rpm"], auth["tpm"])
                if not d["allowed"]:
                    return self._send(429, d, rid, {"Retry-After": str(d["retry_after"])})
                body.setdefault("owner", {})
                try:
                    job_id = plane.submit(body, org_id=org, request_id=rid, tenant_id=tenant)
                except ValueError as e:
                    payload = e.to_payload() if hasattr(e, "to_payload") else {"error": str(e), "code": "BAD_REQUEST"}
                    return self._send(int(getattr(e, "status_code", 400)), payload, rid)
                return self._send(200, {"job_id": job_id, "request_id": rid}, rid)
            if p == "/v1/billing/report":
                try:
                    cost = float(body.get("gpu_hourly_cost", 2.5) or 2.5)
                    limit = int(body.get("limit", 5000) or 5000)
                except (TypeError, ValueError):
                    cost, limit = 2.5, 5000
                return self._send(200, plane.billing_report(org, str(body.get("tenant_id", "") or ""), limit, cost),
                                  rid)
            if p.startswith("/v1/jobs/") and p.endswith("/restore"):
                res = plane.restore(p.split("/")[3], org_id=org, request_id=rid)
                return self._send(200 if res.get("restored") else 400, res, rid)
            return self._send(404, {"error": "not found"}, rid)

    return Handler


def serve(plane, host: str = "127.0.0.1", port: int = 8000, block: bool = True):
    """Start the gateway; returns the server (running in a thread) when ``block`` is False."""
    api_key_salt()  # refuse to start without a configured salt
    rate = float(os.environ.get("KORITH_TENANT_RPS", "50") or 50)
    limiter = RateLimiter()
    bucket = TokenBucket(rate, rate * limiter.burst)
    httpd = ThreadingHTTPServer((host, port), make_handler(plane, limiter, bucket))
    if block:
        httpd.serve_forever()
        return httpd
    threading.Thread(target=httpd.serve_forever, daemon=True).start()
    return httpd


def serve_proxy(upstreams: Dict[str, str], router=None, host: str = "127.0.0.1", port: int = 0,
                timeout_s: float = 300.0, block: bool = False):
    """Reverse proxy in front of OpenAI-compatible servers (``upstreams``: worker id -> base
    URL). ``POST /v1/completions`` and ``/v1/chat/completions`` go to the worker the
    :class:`~.router.ClusterRouter` picks (the one holding the prompt's prefix, else the
    least loaded; its worker ids must be the keys of ``upstreams``), with the choice in the
    ``X-Korith-Route`` response header; every other request goes to the first upstream.
    Reference: platform/gateway/proxy_server.py (a plain pass-through to the router)."""
    import urllib.error
    import urllib.request

    from .control import render_messages

    first = next(iter(upstreams.values()))
    mu = threading.Lock()

    class Proxy(BaseHTTPRequestHandler):
        protocol_version = "HTTP/1.1"

        def log_message(self, *a):
            pass

        def _forward(self, method: str) -> None:
            n = int(self.headers.get("Content-Length", "0") or 0)
            body = self.rfile.read(n) if n > 0 else None
            base, route, wid, added = first, "default", None, 0.0
            path = urlparse(self.path).path
            if method == "POST" and router is not None and path in ("/v1/completions", "/v1/chat/completions"):
                try:
                    req = json.loads(body or b"{}")
                    text = req.get("prompt") if path == "/v1/completions" else render_messages(req.get("messages") or [])
                    if isinstance(text, str) and text:
                        with mu:
                            before = {k: w.load for k, w in router.workers.items()}
                            r = router.submit(text, str(req.get("user", "default")), int(req.get("max_tokens", 16)))
                            added = r.worker.load - before[r.worker.worker_id]
                        if r.worker.worker_id in upstreams:
                            wid, base, route = r.worker.worker_id, upstreams[r.worker.worker_id], r.kind
                        else:
                            with mu:
                                r.worker.load -= added
                except (ValueError, TypeError, RuntimeError):
                    pass  # malformed or unroutable: the default upstream answers
            fwd = urllib.request.Request(base.rstrip("/") + self.path, data=body, method=method)
            for k in ("Content-Type", "Authorization", "X-Request-Id"):
                if self.headers.get(k):
                    fwd.add_header(k, self.headers[k])
            try:
                with urllib.request.urlopen(fwd, timeout=timeout_s) as resp:
                    code, data, ctype = resp.status, resp.read(), resp.headers.get("Content-Type", "application/json")
            except urllib.error.HTTPError as e:
                code, data, ctype = e.code, e.read(), e.headers.get("Content-Type", "application/json")
            except (urllib.error.URLError, OSError) as e:
                code, data, ctype = 502, json.dumps({"error": f"upstream unreachable: {e}"}).encode(), "application/json"
            finally:
                if wid is not None:
                    with mu:  # the request is done: its tokens leave the worker's load
                        w = router.workers[wid]
                        w.load = max(0.0, w.load - added)
            self.send_response(code)
            self.send_header("Content-Type", ctype)
            self.send_header("Content-Length", str(len(data)))
            self.send_header("X-Korith-Route", f"{route}:{wid or 'default'}")
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            self._forward("GET")

        def do_POST(self):
            self._forward("POST")

        def do_DELETE(self):
            self._forward("DELETE")

    httpd = ThreadingHTTPServer((host, port), Proxy)
    if block:
        httpd.serve_forever()
        return httpd
    threading.Thread(target=httpd.serve_forever, daemon=True).start()
    return httpd
