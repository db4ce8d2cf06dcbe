"""Hosted backend: accounts and tokens, keys, metering, dashboard, billing, benchmark data,
the inference proxy (fake upstream) and SSH deployment (fake SSH client)."""
import json
import time
from datetime import timedelta

import httpx
import pytest
from fastapi.testclient import TestClient

from axropus_deploy_b200.saas import Store, create_app, make_token, read_token
from axropus_deploy_b200.saas.store import iso, utcnow


def _upstream():
    seen = []

    def handler(req: httpx.Request):
        seen.append((req.method, str(req.url), req.content, req.headers.get("authorization")))
        if req.url.path == "/v1/models":
            return httpx.Response(200, json={"data": [{"id": "llama3-8b"}]})
        body = json.loads(req.content)
        if body.get("stream"):
            return httpx.Response(200, content=b"data: {\"x\":1}\n\ndata: [DONE]\n\n",
                                  headers={"content-type": "text/event-stream"})
        return httpx.Response(200, json={"choices": [{"text": "hi"}], "echo": body})
    return httpx.MockTransport(handler), seen


@pytest.fixture
def env(tmp_path):
    transport, seen = _upstream()
    bench = tmp_path / "bench"
    bench.mkdir()
    (bench / "BENCH_a.json").write_text(json.dumps({"metric": "output_tok_s", "value": 2900.0, "n_gpus": 1,
                                                    "config": {"model": "llama3-8b"}}) + "\n")
    (bench / "BENCH_b.json").write_text(json.dumps({"metric": "output_tok_s", "value": 2343.1, "n_gpus": 1,
                                                    "impl": "reference", "config": {"model": "llama3-8b"}}) + "\n")
    app = create_app(Store(str(tmp_path / "db.sqlite")), "s3cret", default_upstream="http://node:8000",
                     upstream=transport, bench_dir=str(bench), rate_limit=5, rate_window_s=60,
                     ssh_connect=lambda *a: FakeSSH(), http_get=lambda url: 200, register_wait_s=10)
    return TestClient(app), seen


def _signup(c, email="a@x.io"):
    r = c.post("/api/auth/signup", json={"email": email, "password": "hunter22!", "company_name": "acme"})
    assert r.status_code == 200, r.text
    d = r.json()
    return {"Authorization": "Bearer " + d["access_token"]}, d["api_key"]


def test_tokens_roundtrip_and_reject():
    t = make_token("k", 7, ttl_s=60, now=1000)
    assert read_token("k", t, now=1010) == 7
    with pytest.raises(ValueError):
        read_token("other", t, now=1010)
    with pytest.raises(ValueError):
        read_token("k", t, now=2000)  # expired
    h, b, s = t.split(".")
    with pytest.raises(ValueError):
        read_token("k", h + "." + b[:-2] + "xx." + s, now=1010)


def test_health_auth_keys(env):
    c, _ = env
    assert c.get("/health").json() == {"status": "ok"}
    assert c.get("/health/ready").json() == {"status": "ready"}
    assert c.get("/health").headers["x-frame-options"] == "DENY"
    h, key = _signup(c)
    assert key.startswith("ax-") and len(key) == 35
    assert c.post("/api/auth/signup", json={"email": "a@x.io", "password": "hunter22!"}).status_code == 409
    assert c.post("/api/auth/login", json={"email": "a@x.io", "password": "wrong-pass"}).status_code == 401
    tok = c.post("/api/auth/login", json={"email": "A@x.io", "password": "hunter22!"}).json()["access_token"]
    assert c.get("/api/auth/me", headers={"Authorization": "Bearer " + tok}).json()["email"] == "a@x.io"
    assert c.get("/api/auth/me").status_code == 401
    assert c.get("/api/keys/validate/" + key).json()["tier"] == "trial"
    k2 = c.post("/api/keys/generate", json={"tier": "standard"}, headers=h).json()
    assert k2["status"] == "active" and k2["expires_at"] is None
    assert c.post("/api/keys/generate", json={"tier": "gold"}, headers=h).status_code == 400
    assert len(c.get("/api/keys", headers=h).json()) == 2
    assert c.delete(f"/api/keys/{k2['id']}", headers=h).status_code == 200
    assert c.get("/api/keys/validate/" + k2["key"]).json()["valid"] is False
    h2, _ = _signup(c, "b@x.io")
    assert c.delete(f"/api/keys/{k2['id']}", headers=h2).status_code == 404  # not theirs


def _metric(key, **kw):
    d = {"api_key": key, "timestamp": iso(utcnow()), "tokens_processed": 1000, "amf_hit_rate": 0.5,
         "compute_saved_pct": 0.8, "effective_tps": 2900.0, "baseline_tps": 2343.1, "model_family": "llama3"}
    d.update(kw)
    return d


def test_metrics_dashboard_billing(env):
    c, _ = env
    h, trial = _signup(c)
    std = c.post("/api/keys/generate", json={"tier": "standard"}, headers=h).json()["key"]
    assert c.post("/api/metrics", json=_metric(trial)).status_code == 200
    assert c.post("/api/metrics", json=_metric(std, tokens_processed=3_000_000)).status_code == 200
    assert c.post("/api/metrics", json=_metric(trial, prompt="secret text")).status_code == 400  # not whitelisted
    assert c.post("/api/metrics", json=_metric(trial, model_family="/models/llama.gguf")).status_code == 400
    assert c.post("/api/metrics", json=_metric(trial, adapter_type="10.0.0.1")).status_code == 400
    assert c.post("/api/metrics", json=_metric(trial, amf_hit_rate=1.5)).status_code == 400
    assert c.post("/api/metrics", json=_metric("ax-nope")).status_code == 401
    assert c.post("/api/metrics", json={"api_key": trial}).status_code == 400
    d = c.get("/api/dashboard", headers=h).json()
    assert d["total_tokens_processed"] == 3_001_000 and d["tokens_today"] == 3_001_000
    assert d["status"] == "active" and d["current_effective_tps"] == 2900.0
    assert d["estimated_monthly_savings_usd"] == pytest.approx(3_001_000 * 0.8 * 2.5 / 250_000.0)
    b = c.get("/api/billing/summary", headers=h).json()["current_period"]
    assert b["trial_tokens"] == 1000 and b["standard_tokens"] == 3_000_000
    assert b["billable_tokens"] == 3_000_000 and b["amount_cents"] == 30  # trial tokens within the free allowance
    # a closed month becomes an invoice
    old = iso(utcnow().replace(day=1) - timedelta(days=20))
    assert c.post("/api/metrics", json=_metric(std, timestamp=old, tokens_processed=50_000_000)).status_code == 200
    inv = c.get("/api/billing/invoices", headers=h).json()
    assert len(inv) == 1 and inv[0]["amount_cents"] == 500 and inv[0]["total_tokens"] == 50_000_000
    assert len(c.get("/api/billing/invoices", headers=h).json()) == 1  # not duplicated


def test_benchmarks(env):
    c, _ = env
    runs = c.get("/api/benchmarks/runs", params={"model": "llama3-8b"}).json()
    assert len(runs) == 2
    s = c.get("/api/benchmarks/summary").json()
    assert s[0]["best"] == 2900.0
    m = c.get("/api/benchmarks/mixed").json()["output_tok_s"]
    assert m["reference"] == [2343.1] and m["axropus-b200"] == [2900.0]
    assert "axropus-deploy-b200" in c.get("/").text


def test_inference_proxy_and_rate_limit(env):
    c, seen = env
    _, key = _signup(c)
    bad = c.post("/v1/completions", json={"prompt": "x"}, headers={"Authorization": "Bearer ax-0000"})
    assert bad.status_code == 401
    r = c.post("/v1/completions", json={"prompt": "hello", "max_tokens": 4},
               headers={"Authorization": "Bearer " + key})
    assert r.status_code == 200 and r.json()["echo"]["prompt"] == "hello"
    assert seen[-1][1] == "http://node:8000/v1/completions" and seen[-1][3] == "Bearer " + key
    s = c.post("/v1/chat/completions", json={"messages": [], "stream": True}, headers={"x-api-key": key})
    assert s.headers["content-type"].startswith("text/event-stream") and b"[DONE]" in s.content
    assert c.get("/v1/models", headers={"x-api-key": key}).json()["data"][0]["id"] == "llama3-8b"
    codes = [c.get("/v1/models", headers={"x-api-key": key}).status_code for _ in range(4)]
    assert codes[-1] == 429  # 5 requests per window


class _Out:
    def __init__(self, code, text):
        self.code, self.text = code, text
        self.channel = self

    def recv_exit_status(self):
        return self.code

    def read(self):
        return self.text.encode()


class FakeSSH:
    commands = []

    def exec_command(self, cmd, timeout=None):
        FakeSSH.commands.append(cmd)
        if "--version" in cmd:
            return None, _Out(0, "Python 3.12.3"), _Out(0, "")
        if "nvidia-smi" in cmd:
            return None, _Out(0, "NVIDIA B200, 183359 MiB\nNVIDIA B200, 183359 MiB"), _Out(0, "")
        return None, _Out(0, ""), _Out(0, "")

    def close(self):
        pass


def test_deploy_over_ssh(env):
    c, seen = env
    h, key = _signup(c)
    assert c.post("/api/deploy", json={"host": "gpu1", "username": "ops", "password": "pw"}, headers=h).status_code == 200
    dep = c.get("/api/deploy/status/1", headers=h).json()
    assert dep["deployment"]["runtime"] == "axropus-b200"
    deadline = time.time() + 10
    while time.time() < deadline:
        log = c.get("/api/deploy/status/1", headers=h).json()["log"]
        if any("waiting for the node" in e["message"] for e in log):
            break
        time.sleep(0.02)
    assert c.post("/api/deploy/1/register", json={"api_key": "ax-" + "0" * 32,
                                                   "inference_url": "http://gpu1:8000"}).status_code == 403
    assert c.post("/api/deploy/1/register", json={"api_key": key, "inference_url": "http://gpu1:8000"}).status_code == 200
    while time.time() < deadline:
        st = c.get("/api/deploy/status/1", headers=h).json()
        if st["deployment"]["status"] in ("active", "failed"):
            break
        time.sleep(0.02)
    assert st["deployment"]["status"] == "active", st["log"]
    assert all("pw" != e["message"] and key not in e["message"] for e in st["log"])
    assert any("B200" in e["message"] for e in st["log"])
    assert any("-m axropus_deploy_b200 serve --model llama3-8b" in cmd for cmd in FakeSSH.commands)
    # the websocket replays the whole progress log and closes once the deployment is active
    with c.websocket_connect("/api/deploy/stream/1?token=" + h["Authorization"][7:]) as ws:
        msgs = []
        try:
            while True:
                msgs.append(ws.receive_json())
        except Exception:
            pass
    assert [m["step"] for m in msgs] == [e["step"] for e in st["log"]]
    with pytest.raises(Exception):
        with c.websocket_connect("/api/deploy/stream/1?token=bad") as ws:
            ws.receive_json()
    # the key's traffic now goes to the deployed node
    c.post("/v1/completions", json={"prompt": "x"}, headers={"x-api-key": key})
    assert seen[-1][1] == "http://gpu1:8000/v1/completions"


def test_usage_report_increments():
    from axropus_deploy_b200.saas.agent import usage_report

    prev = {"prefill_tokens": 100, "decode_tokens": 50, "restored_tokens": 0, "local_cached_tokens": 0,
            "cold_prefill_tokens": 100, "amf": {"lookups": 1, "misses": 1}, "spec": {"drafted": 10, "accepted": 5}}
    cur = {"prefill_tokens": 8500, "decode_tokens": 1050, "restored_tokens": 8192, "local_cached_tokens": 8192,
           "cold_prefill_tokens": 8292, "amf": {"lookups": 5, "misses": 2}, "spec": {"drafted": 110, "accepted": 85}}
    r = usage_report(prev, cur, 10.0, 2)
    assert r["tokens_processed"] == 8400 + 1000 and r["prefix_skipped"] == 16384
    assert r["amf_hit_rate"] == pytest.approx(3 / 4) and r["spec_acceptance_rate"] == pytest.approx(0.8)
    assert r["compute_saved_pct"] == pytest.approx(16384 / (16384 + 8192))
    assert r["effective_tps"] == pytest.approx(940.0) and r["gpu_count"] == 2 and r["decode_accelerated"] == 80


def test_agent_registers_and_reports(env):
    from axropus_deploy_b200.saas.agent import Agent

    c, seen = env
    h, key = _signup(c)
    c.post("/api/deploy", json={"host": "gpu2", "username": "ops", "password": "pw"}, headers=h)

    def post_json(url, payload):
        r = c.post("/" + url.split("://", 1)[1].split("/", 1)[1], json=payload)
        if r.status_code >= 400:
            raise RuntimeError(r.text)
        return r.json()

    snaps = iter([{"prefill_tokens": 0, "decode_tokens": 0},
                  {"prefill_tokens": 8320, "decode_tokens": 128, "restored_tokens": 8192, "cold_prefill_tokens": 128}])

    def get_json(url, headers=None):
        if url.endswith("/healthz"):
            return {"ok": True}
        return next(snaps)

    t = iter([0.0, 0.0, 60.0])
    a = Agent("http://backend", key, 1, 8000, "http://gpu2:8000", interval_s=60, post_json=post_json,
              get_json=get_json, clock=lambda: next(t, 60.0))
    assert a.wait_healthy(5) and a.register()
    deadline = time.time() + 10
    while time.time() < deadline:  # the deployment thread sees the registration and goes active
        if c.get("/api/deploy/status/1", headers=h).json()["deployment"]["status"] == "active":
            break
        time.sleep(0.02)
    assert c.get("/api/deploy/status/1", headers=h).json()["deployment"]["inference_url"] == "http://gpu2:8000"
    assert a.report_once() is None  # baseline
    body = a.report_once()
    assert body["tokens_processed"] == 8448 and body["prefix_skipped"] == 8192
    d = c.get("/api/dashboard", headers=h).json()
    assert d["total_tokens_processed"] == 8448 and d["total_prefix_skipped"] == 8192


def test_deploy_starts_the_agent_when_the_backend_url_is_known(tmp_path):
    FakeSSH.commands = []
    app = create_app(Store(str(tmp_path / "db2.sqlite")), "k", ssh_connect=lambda *a: FakeSSH(),
                     http_get=lambda url: 200, register_wait_s=0.2, backend_url="https://backend.example")
    c = TestClient(app)
    h, key = _signup(c, "agent@x.io")
    assert c.post("/api/deploy", json={"host": "gpu3", "username": "ops", "password": "pw"}, headers=h).status_code == 200
    deadline = time.time() + 10
    while time.time() < deadline:
        st = c.get("/api/deploy/status/1", headers=h).json()
        if st["deployment"]["status"] in ("active", "failed"):
            break
        time.sleep(0.02)
    agent = [cmd for cmd in FakeSSH.commands if "axropus_deploy_b200.saas.agent" in cmd]
    assert len(agent) == 1 and "--backend https://backend.example" in agent[0] and "--deployment-id 1" in agent[0]
    assert st["deployment"]["status"] == "failed"  # nobody registered within the 0.2 s given here


def test_proxy_reports_an_unreachable_node(tmp_path):
    def down(req):
        raise httpx.ConnectError("connection refused", request=req)

    app = create_app(Store(str(tmp_path / "db3.sqlite")), "k", default_upstream="http://node:8000",
                     upstream=httpx.MockTransport(down))
    c = TestClient(app)
    _, key = _signup(c, "down@x.io")
    r = c.post("/v1/completions", json={"prompt": "x"}, headers={"x-api-key": key})
    assert r.status_code == 502 and "unavailable" in r.json()["detail"]


def test_enterprise_usage_is_not_billed_per_token(env):
    c, _ = env
    h, _ = _signup(c, "ent@x.io")
    ent = c.post("/api/keys/generate", json={"tier": "enterprise"}, headers=h).json()["key"]
    assert c.post("/api/metrics", json=_metric(ent, tokens_processed=5_000_000)).status_code == 200
    b = c.get("/api/billing/summary", headers=h).json()["current_period"]
    assert b["enterprise_tokens"] == 5_000_000 and b["amount_cents"] == 0 and b["pricing"] == "custom annual pricing"


def test_security_boundaries(env):
    """Cross-account access, forged tokens, injected strings and brute force are refused."""
    c, _ = env
    ha, key_a = _signup(c, "a1@x.io")
    hb, key_b = _signup(c, "b1@x.io")
    assert c.post("/api/deploy", json={"host": "h", "username": "u", "password": "p", "api_key": key_b},
                  headers=ha).status_code == 400  # another account's key
    assert c.post("/api/deploy", json={"host": "h", "username": "u", "password": "p"}, headers=ha).status_code == 200
    assert c.get("/api/deploy/status/1", headers=hb).status_code == 404  # not B's deployment
    forged = make_token("not-the-secret", 1)
    assert c.get("/api/auth/me", headers={"Authorization": "Bearer " + forged}).status_code == 401
    for bad in ("x'; DROP TABLE metrics;--", "../../etc/passwd", "llama<script>"):
        assert c.post("/api/metrics", json=_metric(key_a, sdk_version=bad)).status_code == 400
    assert c.get("/api/keys/validate/' OR 1=1 --").json()["valid"] is False
    codes = [c.post("/api/auth/login", json={"email": "a1@x.io", "password": "wrong-pass"}).status_code
             for _ in range(32)]
    assert codes[0] == 401 and codes[-1] == 429
    r = c.get("/api/keys", headers=ha)
    assert r.headers["x-content-type-options"] == "nosniff" and r.headers["cache-control"] == "no-store"
