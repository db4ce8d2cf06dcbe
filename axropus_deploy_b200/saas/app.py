"""Hosted backend of the framework: accounts, API keys, usage metering, billing, a dashboard,
benchmark data, an OpenAI-compatible inference proxy and deployment of a serving node over SSH.

``create_app`` builds the FastAPI application; every external effect is injectable so the
whole backend runs in tests without a network: ``upstream`` (an ``httpx`` transport to the
serving nodes), ``ssh_connect`` (returns an object with ``exec_command`` and ``close``, by
default a ``paramiko.SSHClient``) and ``http_get`` (the deployment's health probe).

Routes (the reference backend's paths, backend/main.py:50-76 and the routers it includes):

* ``/health``, ``/health/live``, ``/health/ready`` (store reachable)
* ``/api/auth/signup`` (account + a trial key), ``/api/auth/login``, ``/api/auth/me``
* ``/api/keys`` list, ``/api/keys/generate``, ``DELETE /api/keys/{id}`` (revoke),
  ``/api/keys/validate/{key}``
* ``/api/metrics`` -- usage reports from serving nodes: whitelisted fields only, strings
  checked against paths, addresses and model paths so no customer data leaves a node
  (backend/metrics.py:100-160)
* ``/api/dashboard`` -- totals, current rates, today / this week, per-day breakdown, estimated
  monthly savings (backend/dashboard.py:23-126)
* ``/api/billing/summary``, ``/api/billing/invoices`` -- per calendar month: trial tokens free up
  to ``TRIAL_FREE_TOKENS``, standard tokens at ``PRICE_CENTS_PER_MILLION``, enterprise custom;
  savings = tokens x compute saved x GPU cost per token (backend/billing.py:14-123)
* ``/api/benchmarks/summary|runs|mixed`` -- benchmark JSON lines from ``bench_dir``
* ``/v1/completions``, ``/v1/chat/completions``, ``/v1/models`` -- proxied to the key owner's
  active deployment (else ``default_upstream``), rate limited per key
* ``POST /api/deploy``, ``/api/deploy/status/{id}``, ``/api/deploy/{id}/register``, the websocket
  ``/api/deploy/stream/{id}?token=`` (progress messages as they happen) -- install
  and start this framework's server on a customer GPU host over SSH, wait for the node to
  register its URL, probe its health (backend/deploy.py:129-455)
* ``/`` -- a single-page dashboard (static HTML + fetch calls to the routes above)
"""
from __future__ import annotations

import asyncio
import glob
import json
import os
import re
import shlex
import threading
import time
import urllib.request
from collections import defaultdict, deque
from datetime import datetime, timedelta
from typing import Any, Callable, Deque, Dict, List, Optional

import httpx
from fastapi import Depends, FastAPI, HTTPException, Request, WebSocket, WebSocketDisconnect
from fastapi.responses import HTMLResponse, JSONResponse, Response, StreamingResponse
from pydantic import BaseModel, Field

from .store import TIERS, Store, iso, make_token, parse_ts, read_token, utcnow, verify_password

PRICE_CENTS_PER_MILLION = 10.0
TRIAL_FREE_TOKENS = 10_000_000
GPU_COST_PER_HOUR_USD = 2.50
TOKENS_PER_GPU_HOUR = 250_000.0

METRIC_INTS = ("tokens_processed", "interval_seconds", "prefix_skipped", "decode_accelerated", "gpu_count",
               "heartbeat")
METRIC_FLOATS = ("amf_hit_rate", "spec_acceptance_rate", "effective_tps", "baseline_tps", "compute_saved_pct")
METRIC_STRS = ("model_family", "model_size_bucket", "adapter_type", "sdk_version", "license_id")
METRIC_REQUIRED = {"api_key", "timestamp", "tokens_processed"}
METRIC_ALLOWED = METRIC_REQUIRED | set(METRIC_INTS) | set(METRIC_FLOATS) | set(METRIC_STRS)
_SAFE = re.compile(r"[A-Za-z0-9._:+-]{1,128}")
_UNSAFE = re.compile(r"(/|\\|\.\.|~|\b\d{1,3}(\.\d{1,3}){3}\b|\.(gguf|safetensors|bin|pt)\b)", re.I)


class SignupIn(BaseModel):
    email: str = Field(min_length=3, max_length=254)
    password: str = Field(min_length=8, max_length=256)
    company_name: Optional[str] = None


class LoginIn(BaseModel):
    email: str
    password: str


class KeyIn(BaseModel):
    tier: str = "trial"


class DeployIn(BaseModel):
    host: str
    port: int = 22
    username: str
    password: Optional[str] = None
    key_filename: Optional[str] = None
    model_family: str = "llama3"
    model_size: str = "8b"
    runtime: str = "axropus-b200"
    api_key: Optional[str] = None
    python_bin: str = "python3"
    serve_port: int = 8000


class RegisterIn(BaseModel):
    api_key: str
    inference_url: str


class RateLimiter:
    """Sliding-window request counter per key."""

    def __init__(self):
        self.hits: Dict[str, Deque[float]] = defaultdict(deque)
        self.mu = threading.Lock()

    def allow(self, key: str, limit: int, window_s: float) -> bool:
        now = time.monotonic()
        with self.mu:
            q = self.hits[key]
            while q and q[0] <= now - window_s:
                q.popleft()
            if len(q) >= limit:
                return False
            q.append(now)
            return True


def _period(now: datetime):
    start = now.replace(day=1, hour=0, minute=0, second=0, microsecond=0)
    nxt = (start + timedelta(days=32)).replace(day=1)
    return start, nxt - timedelta(seconds=1)


def _paramiko_connect(host: str, port: int, username: str, password: Optional[str], key_filename: Optional[str]):
    import paramiko

    c = paramiko.SSHClient()
    c.set_missing_host_key_policy(paramiko.AutoAddPolicy())
    c.connect(host, port=port, username=username, password=password, key_filename=key_filename, timeout=20)
    return c


def _http_get(url: str, timeout: float = 10.0) -> int:
    with urllib.request.urlopen(url, timeout=timeout) as r:
        return int(r.status)


def create_app(store: Optional[Store] = None, secret: Optional[str] = None, *, default_upstream: str = "",
               upstream: Optional[httpx.AsyncBaseTransport] = None, ssh_connect: Callable = _paramiko_connect,
               http_get: Callable[[str], int] = _http_get, bench_dir: Optional[str] = None,
               rate_limit: int = 600, rate_window_s: float = 60.0, register_wait_s: float = 600.0,
               install_cmd: str = "{py} -m pip install --upgrade axropus-deploy-b200",
               backend_url: Optional[str] = None) -> FastAPI:
    """``backend_url``: this backend's address as the deployed nodes reach it; when set, a
    deployment also starts the node agent (``saas/agent.py``), which registers the node and
    reports its usage."""
    store = store or Store(os.environ.get("AXROPUS_SAAS_DB", ":memory:"))
    backend_url = backend_url if backend_url is not None else os.environ.get("AXROPUS_SAAS_PUBLIC_URL", "")
    secret = secret or os.environ.get("AXROPUS_SAAS_SECRET") or os.urandom(32).hex()
    limiter = RateLimiter()
    progress: Dict[int, List[Dict[str, Any]]] = defaultdict(list)
    progress_mu = threading.Lock()
    app = FastAPI(title="axropus-deploy-b200 backend")
    app.state.store = store

    @app.middleware("http")
    async def headers(request: Request, call_next):
        resp = await call_next(request)
        resp.headers["X-Content-Type-Options"] = "nosniff"
        resp.headers["X-Frame-Options"] = "DENY"
        resp.headers["Referrer-Policy"] = "no-referrer"
        resp.headers["Cache-Control"] = "no-store"
        return resp

    # ---------------------------------------------------------------- health
    @app.get("/health")
    def health():
        return {"status": "ok"}

    @app.get("/health/live")
    def live():
        return {"status": "live"}

    @app.get("/health/ready")
    def ready():
        return {"status": "ready"} if store.ping() else JSONResponse({"status": "not_ready"}, status_code=503)

    # ---------------------------------------------------------------- accounts
    def customer(request: Request) -> Dict[str, Any]:
        auth = request.headers.get("authorization", "")
        if not auth.lower().startswith("bearer "):
            raise HTTPException(401, "missing bearer token")
        try:
            cid = read_token(secret, auth[7:].strip())
        except ValueError as e:
            raise HTTPException(401, f"invalid token: {e}") from None
        row = store.one("SELECT id, email, company_name, created_at FROM customers WHERE id=?", (cid,))
        if row is None:
            raise HTTPException(401, "unknown customer")
        return row

    @app.post("/api/auth/signup")
    def signup(body: SignupIn, request: Request):
        if not limiter.allow("signup:" + (request.client.host if request.client else "-"), 10, 3600):
            raise HTTPException(429, "too many signups")
        if "@" not in body.email:
            raise HTTPException(400, "invalid email")
        if store.one("SELECT id FROM customers WHERE email=?", (body.email.lower(),)):
            raise HTTPException(409, "email already registered")
        cid = store.add_customer(body.email, body.password, body.company_name)
        key = store.add_key(cid, "trial")
        return {"customer_id": cid, "access_token": make_token(secret, cid), "token_type": "bearer",
                "api_key": key["key"], "expires_at": key["expires_at"]}

    @app.post("/api/auth/login")
    def login(body: LoginIn, request: Request):
        if not limiter.allow("login:" + (request.client.host if request.client else "-"), 30, 300):
            raise HTTPException(429, "too many attempts")
        row = store.one("SELECT id, password_hash FROM customers WHERE email=?", (body.email.lower(),))
        if row is None or not verify_password(body.password, row["password_hash"]):
            raise HTTPException(401, "invalid credentials")
        return {"access_token": make_token(secret, row["id"]), "token_type": "bearer"}

    @app.get("/api/auth/me")
    def me(c=Depends(customer)):
        return c

    # ---------------------------------------------------------------- keys
    @app.get("/api/keys")
    def keys(c=Depends(customer)):
        return store.q("SELECT id, key, status, tier, created_at, expires_at FROM api_keys WHERE customer_id=? "
                       "ORDER BY id", (c["id"],))

    @app.post("/api/keys/generate")
    def gen_key(body: KeyIn, c=Depends(customer)):
        if body.tier not in TIERS:
            raise HTTPException(400, f"tier must be one of {list(TIERS)}")
        row = store.add_key(c["id"], body.tier)
        return {k: row[k] for k in ("id", "key", "status", "tier", "created_at", "expires_at")}

    @app.delete("/api/keys/{key_id}")
    def revoke(key_id: int, c=Depends(customer)):
        row = store.one("SELECT * FROM api_keys WHERE id=? AND customer_id=?", (key_id, c["id"]))
        if row is None:
            raise HTTPException(404, "no such key")
        store.exec("UPDATE api_keys SET status='revoked', expires_at=? WHERE id=?", (iso(utcnow()), key_id))
        return {"revoked": key_id}

    @app.get("/api/keys/validate/{key_value}")
    def validate(key_value: str):
        row = store.active_key(key_value)
        if row is None:
            return {"valid": False, "tier": None, "customer_id": None}
        return {"valid": True, "tier": row["tier"], "customer_id": row["customer_id"]}

    # ---------------------------------------------------------------- metrics
    def _clean_str(name: str, v: Any) -> Optional[str]:
        if v is None:
            return None
        s = str(v).strip()
        if not s:
            return None
        if _SAFE.fullmatch(s) is None or _UNSAFE.search(s):
            raise HTTPException(400, f"{name} contains unsafe content")
        return s

    @app.post("/api/metrics")
    def ingest(payload: Dict[str, Any]):
        extra = set(payload) - METRIC_ALLOWED
        if extra:
            raise HTTPException(400, "non-whitelisted fields: " + ", ".join(sorted(extra)))
        missing = METRIC_REQUIRED - set(payload)
        if missing:
            raise HTTPException(400, "missing fields: " + ", ".join(sorted(missing)))
        key = store.active_key(str(payload["api_key"]))
        if key is None:
            raise HTTPException(401, "invalid or expired api_key")
        try:
            ts = parse_ts(str(payload["timestamp"]))
            vals = {k: int(payload.get(k, 0) or 0) for k in METRIC_INTS}
            vals.update({k: float(payload.get(k, 0.0) or 0.0) for k in METRIC_FLOATS})
        except (TypeError, ValueError):
            raise HTTPException(400, "non-numeric or malformed field") from None
        if any(v < 0 for v in vals.values()) or not 0 <= vals["amf_hit_rate"] <= 1 \
                or not 0 <= vals["spec_acceptance_rate"] <= 1 or not 0 <= vals["compute_saved_pct"] <= 1:
            raise HTTPException(400, "field out of range")
        vals.setdefault("interval_seconds", 60)
        strs = {k: _clean_str(k, payload.get(k)) for k in METRIC_STRS}
        cols = ["api_key_id", "timestamp"] + list(vals) + list(strs)
        mid = store.exec(f"INSERT INTO metrics ({','.join(cols)}) VALUES ({','.join('?' * len(cols))})",
                         [key["id"], iso(ts)] + list(vals.values()) + list(strs.values()))
        return {"accepted": True, "id": mid}

    def _usage(cid: int, since: Optional[datetime] = None, until: Optional[datetime] = None):
        sql = ("SELECT m.*, k.tier FROM metrics m JOIN api_keys k ON k.id = m.api_key_id WHERE k.customer_id=?")
        args: List[Any] = [cid]
        if since is not None:
            sql += " AND m.timestamp >= ?"
            args.append(iso(since))
        if until is not None:
            sql += " AND m.timestamp <= ?"
            args.append(iso(until))
        return store.q(sql + " ORDER BY m.timestamp", args)

    def _savings_usd(rows) -> float:
        return sum(r["tokens_processed"] * r["compute_saved_pct"] * (GPU_COST_PER_HOUR_USD / TOKENS_PER_GPU_HOUR)
                   for r in rows)

    # ---------------------------------------------------------------- dashboard
    @app.get("/api/dashboard")
    def dashboard(c=Depends(customer)):
        rows = _usage(c["id"])
        now = utcnow()
        day0 = now.replace(hour=0, minute=0, second=0)
        out = {"total_tokens_processed": 0, "total_prefix_skipped": 0, "total_decode_accelerated": 0,
               "current_amf_hit_rate": 0.0, "current_spec_acceptance_rate": 0.0, "current_effective_tps": 0.0,
               "current_baseline_tps": 0.0, "current_compute_saved_pct": 0.0, "estimated_monthly_savings_usd": 0.0,
               "tokens_today": 0, "tokens_this_week": 0, "daily_breakdown": [], "status": "inactive"}
        if not rows:
            return out
        latest = rows[-1]
        days: Dict[str, List[Dict[str, Any]]] = defaultdict(list)
        for r in rows:
            days[r["timestamp"][:10]].append(r)
        last30 = [r for r in rows if parse_ts(r["timestamp"]) >= now - timedelta(days=30)]
        out.update({
            "total_tokens_processed": sum(r["tokens_processed"] for r in rows),
            "total_prefix_skipped": sum(r["prefix_skipped"] for r in rows),
            "total_decode_accelerated": sum(r["decode_accelerated"] for r in rows),
            "current_amf_hit_rate": latest["amf_hit_rate"], "current_spec_acceptance_rate": latest["spec_acceptance_rate"],
            "current_effective_tps": latest["effective_tps"], "current_baseline_tps": latest["baseline_tps"],
            "current_compute_saved_pct": latest["compute_saved_pct"],
            "estimated_monthly_savings_usd": round(_savings_usd(last30), 6),
            "tokens_today": sum(r["tokens_processed"] for r in rows if parse_ts(r["timestamp"]) >= day0),
            "tokens_this_week": sum(r["tokens_processed"] for r in rows
                                    if parse_ts(r["timestamp"]) >= now - timedelta(days=7)),
            "daily_breakdown": [{"date": d, "tokens": sum(r["tokens_processed"] for r in rs),
                                 "savings_pct": sum(r["compute_saved_pct"] for r in rs) / len(rs)}
                                for d, rs in sorted(days.items())][-30:],
            "status": "active" if parse_ts(latest["timestamp"]) >= now - timedelta(minutes=10) else "inactive",
        })
        return out

    # ---------------------------------------------------------------- billing
    def _bill(rows) -> Dict[str, Any]:
        by = {t: sum(r["tokens_processed"] for r in rows if r["tier"] == t) for t in TIERS}
        billable = max(0, by["trial"] - TRIAL_FREE_TOKENS) + by["standard"]
        cents = int(round(billable / 1e6 * PRICE_CENTS_PER_MILLION))
        savings = _savings_usd(rows)
        return {"total_tokens": sum(by.values()), "trial_tokens": by["trial"], "standard_tokens": by["standard"],
                "enterprise_tokens": by["enterprise"], "billable_tokens": billable, "amount_cents": cents,
                "estimated_savings_usd": round(savings, 6),
                "roi": round(savings / (cents / 100.0), 4) if cents else None,
                "pricing": ("custom annual pricing" if by["enterprise"] and not billable
                            else f"${PRICE_CENTS_PER_MILLION / 100:.2f} per million tokens")}

    @app.get("/api/billing/summary")
    def billing(c=Depends(customer)):
        start, end = _period(utcnow())
        return {"current_period": {"start": str(start.date()), "end": str(end.date()),
                                   **_bill(_usage(c["id"], start, end))}}

    @app.get("/api/billing/invoices")
    def invoices(c=Depends(customer)):
        """One invoice per closed calendar month with usage (created on first request)."""
        rows = _usage(c["id"])
        now_start, _ = _period(utcnow())
        months = sorted({r["timestamp"][:7] for r in rows})
        for m in months:
            start = datetime.fromisoformat(m + "-01")
            if start >= now_start:
                continue
            if store.one("SELECT id FROM invoices WHERE customer_id=? AND period_start=?", (c["id"], str(start.date()))):
                continue
            s, e = _period(start)
            b = _bill(_usage(c["id"], s, e))
            store.exec("INSERT INTO invoices (customer_id, period_start, period_end, total_tokens, amount_cents, "
                       "status, created_at) VALUES (?,?,?,?,?,?,?)",
                       (c["id"], str(s.date()), str(e.date()), b["total_tokens"], b["amount_cents"],
                        "pending" if b["amount_cents"] else "paid", iso(utcnow())))
        return store.q("SELECT * FROM invoices WHERE customer_id=? ORDER BY period_start", (c["id"],))

    # ---------------------------------------------------------------- benchmarks
    def _runs() -> List[Dict[str, Any]]:
        runs = []
        for path in sorted(glob.glob(os.path.join(bench_dir, "*.json*"))) if bench_dir else []:
            with open(path) as f:
                for line in f:
                    line = line.strip()
                    if line.startswith("{"):
                        try:
                            d = json.loads(line)
                        except ValueError:
                            continue
                        if "metric" in d and "value" in d:
                            d["source"] = os.path.basename(path)
                            runs.append(d)
        return runs

    @app.get("/api/benchmarks/runs")
    def bench_runs(metric: Optional[str] = None, model: Optional[str] = None):
        rs = _runs()
        if metric:
            rs = [r for r in rs if r["metric"] == metric]
        if model:
            rs = [r for r in rs if (r.get("config") or {}).get("model") == model]
        return rs

    @app.get("/api/benchmarks/summary")
    def bench_summary():
        best: Dict[str, Dict[str, Any]] = {}
        for r in _runs():
            key = f"{r['metric']}|{(r.get('config') or {}).get('model', '')}|{r.get('n_gpus', 1)}"
            hib = r.get("higher_is_better", True)
            cur = best.get(key)
            if cur is None or (r["value"] > cur["value"]) == hib:
                best[key] = r
        return [{"metric": r["metric"], "model": (r.get("config") or {}).get("model"), "n_gpus": r.get("n_gpus", 1),
                 "best": r["value"], "unit": r.get("unit"), "vs_baseline": r.get("vs_baseline"), "source": r["source"]}
                for r in best.values()]

    @app.get("/api/benchmarks/mixed")
    def bench_mixed():
        """Runs by implementation (this framework against the reference arm) for each metric."""
        out: Dict[str, Dict[str, List[float]]] = defaultdict(lambda: defaultdict(list))
        for r in _runs():
            out[r["metric"]][r.get("impl", "axropus-b200")].append(r["value"])
        return {m: dict(v) for m, v in out.items()}

    # ---------------------------------------------------------------- inference proxy
    def _api_key(request: Request) -> Dict[str, Any]:
        auth = request.headers.get("authorization", "")
        value = auth[7:].strip() if auth.lower().startswith("bearer ") else request.headers.get("x-api-key", "")
        row = store.active_key(value)
        if row is None:
            raise HTTPException(401, "invalid or expired api key")
        if not limiter.allow("key:" + value, rate_limit, rate_window_s):
            raise HTTPException(429, "rate limit exceeded")
        return row

    def _upstream_url(key: Dict[str, Any]) -> str:
        dep = store.one("SELECT inference_url FROM deployments WHERE customer_id=? AND status='active' AND "
                        "inference_url IS NOT NULL ORDER BY id DESC", (key["customer_id"],))
        url = dep["inference_url"] if dep else default_upstream
        if not url:
            raise HTTPException(503, "no active deployment")
        return url.rstrip("/")

    async def _proxy(request: Request, path: str):
        key = _api_key(request)
        url = _upstream_url(key) + path
        body = await request.body()
        client = httpx.AsyncClient(transport=upstream, timeout=600.0)
        # the node was started with the owner's key (``axropus serve --api-key``): present it
        req = client.build_request(request.method, url, content=body,
                                   headers={"content-type": request.headers.get("content-type", "application/json"),
                                            "authorization": "Bearer " + key["key"]})
        try:
            resp = await client.send(req, stream=True)
        except httpx.HTTPError as e:
            await client.aclose()
            raise HTTPException(502, f"serving node unavailable: {type(e).__name__}") from None
        ctype = resp.headers.get("content-type", "application/json")
        if ctype.startswith("text/event-stream"):
            async def gen():
                try:
                    async for chunk in resp.aiter_bytes():
                        yield chunk
                finally:
                    await resp.aclose()
                    await client.aclose()
            return StreamingResponse(gen(), status_code=resp.status_code, media_type=ctype)
        data = await resp.aread()
        await resp.aclose()
        await client.aclose()
        return Response(data, status_code=resp.status_code, media_type=ctype)

    @app.post("/v1/completions")
    async def completions(request: Request):
        return await _proxy(request, "/v1/completions")

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        return await _proxy(request, "/v1/chat/completions")

    @app.get("/v1/models")
    async def models(request: Request):
        return await _proxy(request, "/v1/models")

    # ---------------------------------------------------------------- deployment over SSH
    def _log(dep_id: int, step: int, state: str, message: str, progress_frac: float, mask: List[str]) -> None:
        for s in mask:
            if s:
                message = message.replace(s, "***")
        with progress_mu:
            progress[dep_id].append({"step": step, "status": state, "message": message,
                                     "progress": round(progress_frac, 3), "ts": time.time()})

    def _run(ssh, cmd: str, timeout: int = 240):
        _, out, err = ssh.exec_command(cmd, timeout=timeout)
        code = out.channel.recv_exit_status()
        return code, out.read().decode(errors="replace"), err.read().decode(errors="replace")

    def _deploy_task(dep_id: int, body: DeployIn, key_value: str) -> None:
        mask = [body.password or "", key_value]
        store.exec("UPDATE deployments SET status='deploying' WHERE id=?", (dep_id,))
        ssh = None
        try:
            _log(dep_id, 1, "running", f"connecting to {body.username}@{body.host}:{body.port}", 0.05, mask)
            ssh = ssh_connect(body.host, body.port, body.username, body.password, body.key_filename)
            _log(dep_id, 1, "success", "connected", 0.10, mask)
            py = shlex.quote(body.python_bin)
            code, out, err = _run(ssh, f"{py} --version")
            m = re.search(r"(\d+)\.(\d+)", out + err)
            if code != 0 or m is None or (int(m.group(1)), int(m.group(2))) < (3, 10):
                raise RuntimeError(f"python 3.10+ required, found {(out + err).strip() or 'none'}")
            _log(dep_id, 2, "success", (out + err).strip(), 0.20, mask)
            code, gpu, _ = _run(ssh, "nvidia-smi --query-gpu=name,memory.total --format=csv,noheader")
            if code != 0 or not gpu.strip():
                raise RuntimeError("no NVIDIA GPU visible on the host")
            _log(dep_id, 3, "success", "GPUs: " + "; ".join(x.strip() for x in gpu.strip().splitlines()), 0.30, mask)
            code, out, err = _run(ssh, install_cmd.format(py=py), timeout=1800)
            if code != 0:
                raise RuntimeError("install failed: " + (err or out)[-400:])
            _log(dep_id, 4, "success", "framework installed", 0.55, mask)
            model = shlex.quote(f"{body.model_family}-{body.model_size}")
            start = (f"nohup {py} -m axropus_deploy_b200 serve --model {model} --host 0.0.0.0 "
                     f"--port {int(body.serve_port)} --api-key {shlex.quote(key_value)} > axropus_server.log 2>&1 &")
            code, out, err = _run(ssh, start)
            if code != 0:
                raise RuntimeError("server start failed: " + (err or out)[-400:])
            if backend_url:
                agent = (f"nohup {py} -m axropus_deploy_b200.saas.agent --backend {shlex.quote(backend_url)} "
                         f"--deployment-id {dep_id} --api-key {shlex.quote(key_value)} --port {int(body.serve_port)} "
                         f"--model-family {shlex.quote(body.model_family)} > axropus_agent.log 2>&1 &")
                code, out, err = _run(ssh, agent)
                if code != 0:
                    raise RuntimeError("agent start failed: " + (err or out)[-400:])
            _log(dep_id, 5, "success", "server started; waiting for the node to register", 0.70, mask)
            url = None
            t_end = time.monotonic() + register_wait_s
            while time.monotonic() < t_end:
                row = store.one("SELECT inference_url FROM deployments WHERE id=?", (dep_id,))
                if row and row["inference_url"]:
                    url = row["inference_url"]
                    break
                time.sleep(0.05)
            if url is None:
                raise RuntimeError("node did not register in time")
            _log(dep_id, 6, "success", f"node registered at {url}", 0.85, mask)
            st = http_get(url.rstrip("/") + "/healthz")
            if st != 200:
                raise RuntimeError(f"health probe returned {st}")
            store.exec("UPDATE deployments SET status='active', deployed_at=? WHERE id=?", (iso(utcnow()), dep_id))
            _log(dep_id, 7, "success", "deployment active", 1.0, mask)
        except Exception as e:
            store.exec("UPDATE deployments SET status='failed' WHERE id=?", (dep_id,))
            _log(dep_id, 99, "failed", f"deployment failed: {e}", 1.0, mask)
        finally:
            if ssh is not None:
                try:
                    ssh.close()
                except Exception:
                    pass

    @app.post("/api/deploy")
    def deploy(body: DeployIn, c=Depends(customer)):
        if body.runtime != "axropus-b200":
            raise HTTPException(400, "runtime must be axropus-b200")
        if not (body.password or body.key_filename):
            raise HTTPException(400, "password or key_filename required")
        if body.api_key:
            key = store.active_key(body.api_key)
            if key is None or key["customer_id"] != c["id"]:
                raise HTTPException(400, "api_key is not an active key of this account")
        else:
            key = store.one("SELECT * FROM api_keys WHERE customer_id=? AND status!='revoked' ORDER BY id DESC",
                            (c["id"],))
            key = store.active_key(key["key"]) if key else None
            if key is None:
                raise HTTPException(400, "no active api key")
        dep_id = store.exec("INSERT INTO deployments (customer_id, api_key_id, runtime, model_family, model_size, "
                            "status) VALUES (?,?,?,?,?,'pending')",
                            (c["id"], key["id"], body.runtime, body.model_family, body.model_size))
        threading.Thread(target=_deploy_task, args=(dep_id, body, key["key"]), daemon=True,
                         name=f"deploy-{dep_id}").start()
        return {"deployment_id": dep_id, "status": "pending"}

    @app.get("/api/deploy/status/{dep_id}")
    def deploy_status(dep_id: int, since: int = 0, c=Depends(customer)):
        row = store.one("SELECT * FROM deployments WHERE id=? AND customer_id=?", (dep_id, c["id"]))
        if row is None:
            raise HTTPException(404, "no such deployment")
        with progress_mu:
            log = progress[dep_id][since:]
        return {"deployment": row, "log": log, "next": since + len(log)}

    @app.websocket("/api/deploy/stream/{dep_id}")
    async def deploy_stream(ws: WebSocket, dep_id: int):
        """Progress messages of a deployment as they are logged, until it is active or failed
        (browsers cannot set headers on a websocket: the access token comes as ``?token=``)."""
        try:
            cid = read_token(secret, ws.query_params.get("token", ""))
        except ValueError:
            await ws.close(code=4401)
            return
        if store.one("SELECT id FROM deployments WHERE id=? AND customer_id=?", (dep_id, cid)) is None:
            await ws.close(code=4404)
            return
        await ws.accept()
        cursor = 0
        try:
            while True:
                with progress_mu:
                    msgs = progress[dep_id][cursor:]
                for m in msgs:
                    await ws.send_json(m)
                cursor += len(msgs)
                row = store.one("SELECT status FROM deployments WHERE id=?", (dep_id,))
                if not msgs and row["status"] in ("active", "failed"):
                    break
                await asyncio.sleep(0.05)
        except WebSocketDisconnect:
            return
        await ws.close()

    @app.post("/api/deploy/{dep_id}/register")
    def register(dep_id: int, body: RegisterIn):
        key = store.active_key(body.api_key)
        row = store.one("SELECT * FROM deployments WHERE id=?", (dep_id,))
        if key is None or row is None or row["api_key_id"] != key["id"]:
            raise HTTPException(403, "key does not own this deployment")
        if not re.fullmatch(r"https?://[A-Za-z0-9.\-\[\]:]+(/[A-Za-z0-9._~/-]*)?", body.inference_url):
            raise HTTPException(400, "invalid inference_url")
        store.exec("UPDATE deployments SET inference_url=? WHERE id=?", (body.inference_url, dep_id))
        return {"registered": dep_id}

    # ---------------------------------------------------------------- dashboard page
    @app.get("/", response_class=HTMLResponse)
    def index():
        return DASHBOARD_HTML

    return app


DASHBOARD_HTML = """<!doctype html>
<html><head><meta charset="utf-8"><title>axropus-deploy-b200</title>
<style>body{font:14px system-ui,sans-serif;margin:2em;max-width:60em}table{border-collapse:collapse}
td,th{border:1px solid #ccc;padding:4px 8px}section{margin:1.5em 0}.hide{display:none}</style></head>
<body><h1>axropus-deploy-b200</h1>
<section id="auth"><h2>Sign in</h2><input id="email" placeholder="email"> <input id="pw" type="password"
 placeholder="password"> <button onclick="login()">Log in</button> <button onclick="signup()">Sign up</button>
<div id="msg"></div></section>
<section id="app" class="hide"><h2>Usage</h2><table id="usage"></table>
<h2>Billing (this month)</h2><table id="bill"></table>
<h2>API keys</h2><table id="keys"></table><button onclick="newKey()">New key</button>
<h2>Benchmarks</h2><table id="bench"></table></section>
<script>
let tok = null;
const H = () => ({'Content-Type': 'application/json', 'Authorization': 'Bearer ' + tok});
async function call(path, opt) { const r = await fetch(path, opt || {headers: H()}); return r.json(); }
function table(id, obj) {
  const rows = Array.isArray(obj) ? obj : Object.entries(obj).map(([k, v]) => ({field: k,
      value: typeof v === 'object' ? JSON.stringify(v) : v}));
  if (!rows.length) { document.getElementById(id).innerHTML = '<tr><td>none</td></tr>'; return; }
  const cols = Object.keys(rows[0]);
  const esc = s => String(s).replace(/[&<>]/g, c => ({'&': '&amp;', '<': '&lt;', '>': '&gt;'}[c]));
  document.getElementById(id).innerHTML = '<tr>' + cols.map(c => '<th>' + esc(c) + '</th>').join('') + '</tr>' +
    rows.map(r => '<tr>' + cols.map(c => '<td>' + esc(r[c]) + '</td>').join('') + '</tr>').join('');
}
async function auth(path) {
  const r = await call(path, {method: 'POST', headers: {'Content-Type': 'application/json'},
    body: JSON.stringify({email: email.value, password: pw.value})});
  if (!r.access_token) { msg.textContent = JSON.stringify(r.detail || r); return; }
  tok = r.access_token; document.getElementById('auth').classList.add('hide');
  document.getElementById('app').classList.remove('hide'); refresh();
}
const login = () => auth('/api/auth/login'), signup = () => auth('/api/auth/signup');
async function newKey() { await call('/api/keys/generate', {method: 'POST', headers: H(),
  body: JSON.stringify({tier: 'standard'})}); refresh(); }
async function refresh() {
  const d = await call('/api/dashboard'); delete d.daily_breakdown; table('usage', d);
  table('bill', (await call('/api/billing/summary')).current_period);
  table('keys', await call('/api/keys'));
  table('bench', await call('/api/benchmarks/summary'));
}
</script></body></html>
"""
