"""Control plane on CPU: ledger, economics, adapters + worker + control plane over a tiny
engine with an AMF pool, the HTTP gateway (auth, limits, job lifecycle), node registry,
snapshot index and node-to-node snapshot transfer, runtime governance and the
Dynamo-style scoring / storage / event components."""
import json
import os
import time
import urllib.error
import urllib.request

import pytest
import torch

from axropus_deploy_b200.cluster.economics import TenantMeter, estimate_savings, write_report
from axropus_deploy_b200.cluster.ledger import SqliteLedger
from axropus_deploy_b200.cluster.observability import ArtifactStore, MetricsRegistry


def _engine(num_blocks=160):
    from axropus_deploy_b200.amf import AmfManager, G1Pool
    from axropus_deploy_b200.engine import EngineConfig, LLMEngine
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel

    model = LlamaModel(get_config("tiny"), "cpu", seed=0)
    c = model.cfg
    pool = G1Pool(c.num_layers, c.num_kv_heads, c.head_dim, "raw", slots_per_shard=64)
    return LLMEngine(model, EngineConfig(num_blocks=num_blocks, max_model_len=1024), AmfManager(raw_pool=pool))


def _plane(tmp_path, node="node-a", ledger=None, nodes=None):
    from axropus_deploy_b200.cluster.adapters import AdapterRegistry
    from axropus_deploy_b200.cluster.control import ControlPlane
    from axropus_deploy_b200.cluster.nodes import SnapshotIndex
    from axropus_deploy_b200.cluster.runtime import DecodeCache
    from axropus_deploy_b200.cluster.worker import ClusterWorker

    ledger = ledger or SqliteLedger(str(tmp_path / "ledger.db"))
    index = SnapshotIndex(ledger, tier_roots={"ram": str(tmp_path / node / "ram")})
    art = ArtifactStore(tmp_path / node / "ram")
    w = ClusterWorker(f"{node}-w0", node, AdapterRegistry(_engine()), ledger, art, snapshot_index=index,
                      node_registry=nodes, decode_cache=DecodeCache(), metrics=MetricsRegistry(),
                      link_gbps=10.0, rtt_ms=0.1)
    return ControlPlane(ledger, {w.worker_id: w}, node_id=node, snapshot_index=index, node_registry=nodes,
                        metrics=w.metrics), w, index


PROMPT = "system: you are a careful assistant. " * 14  # 518 bytes: the 512-token shared prefix


def test_ledger_roundtrip(tmp_path):
    led = SqliteLedger(str(tmp_path / "l.db"))
    led.insert_job("j1", "2026-01-01T00:00:00Z", {"prompt": "x", "max_tokens": 4}, {"m": 1}, "ph", "fp", "idem-1",
                   "queued", "org1")
    assert led.get_job("j1")["status"] == "queued" and led.verify_job("j1")
    assert led.find_job_by_idempotency("idem-1", "org1") == "j1" and led.find_job_by_fingerprint("fp") == "j1"
    led.update_status("j1", "succeeded")
    led.insert_run("r1", "j1", "a", "b", 0, "m", "e", "o", "l", "org1")
    assert led.get_latest_run("j1")["run_id"] == "r1"
    for i in range(10):
        led.upsert_snapshot_location("fp", f"s{i}", "org1", f"n{i}", None, f"/p{i}", 10, "t", f"2026-01-01T00:00:{i:02d}Z")
    assert led.prune_snapshot_locations(4) == 6 and len(led.list_snapshot_locations("fp", "org1")) == 4
    led.create_api_key("k1", "h1", "org1", "t", 100, 10, "{}")
    assert led.get_api_key_by_hash("h1")["org_id"] == "org1" and led.revoke_api_key("k1", "t2")
    assert not led.revoke_api_key("k1", "t3")


def test_economics(tmp_path):
    m = {"perf": {"total_ms": 100.0, "prefill_ms": 10.0, "decode_ms": 90.0},
         "amf": {"decision": "hit", "saved_ms": 300.0}, "spec": {"saved_ms": 20.0}}
    s = estimate_savings(m, 3.6)
    assert s["saved_ms"] == 320.0 and abs(s["cost_saved_usd"] - 320 * 1e-6) < 1e-12
    t = TenantMeter("t1")
    t.accumulate(m)
    t.accumulate({"perf": {"total_ms": 400.0}, "amf": {"decision": "miss"}})
    sm = t.summary(3.6)
    assert sm["amf_hit_rate"] == 0.5 and abs(sm["savings_pct"] - 100 * 320 / 820) < 1e-9
    led = SqliteLedger(str(tmp_path / "l.db"))
    mp = tmp_path / "m.json"
    mp.write_text(json.dumps(m))
    led.insert_job("j", "t", {"prompt": "p", "tenant_id": "t1"}, {}, "h", "f", None, "succeeded")
    led.insert_run("r", "j", "a", "b", 0, str(mp), "", "", "")
    for ext in ("json", "md", "pdf"):
        rep = write_report(led, tmp_path / f"rep.{ext}", 2.5, targets=[0.5, 0.9])
    assert (tmp_path / "rep.pdf").read_bytes().startswith(b"%PDF-1.4") and b"%%EOF" in (tmp_path / "rep.pdf").read_bytes()
    assert rep["targets"]["targets"][0]["met"] and not rep["targets"]["targets"][1]["met"]


def test_control_plane_jobs_hits_and_kpis(tmp_path):
    plane, w, index = _plane(tmp_path)
    j1 = plane.submit({"prompt": PROMPT + "question one?", "max_tokens": 4, "amf_prefix_len": 512}, org_id="org1",
                       tenant_id="t1")
    r1 = w.drain()[0]
    assert r1["exit_code"] == 0 and r1["amf"]["decision"] == "miss" and r1["lane"] == "MISS"
    job = plane.get_job(j1, "org1")
    assert job["status"] == "succeeded" and job["immutable"] and len(job["output_text"]) > 0
    # the cold run captured its prefix and exported a snapshot with a valid sidecar
    snap = plane.ledger.get_snapshot_for_job(j1)
    assert snap is not None and os.path.exists(snap["snapshot_path"] + ".meta.json")
    fp = job["fingerprint_hash"]
    assert index.get_locations(fp, "org1")[0]["storage_tier"] == "ram"
    # same prefix, new question: routed as a HIT, served from the live prefix cache / pool
    w.adapters.engine.evict_live_cache()
    j2 = plane.submit({"prompt": PROMPT + "question two!", "max_tokens": 4, "amf_prefix_len": 512}, org_id="org1",
                       tenant_id="t1")
    r2 = w.drain()[0]
    assert r2["lane"] == "HIT" and r2["amf"]["decision"] == "hit" and r2["amf"]["restored_tokens"] > 0
    # identical deterministic job: decode cache
    plane.submit({"prompt": PROMPT + "question two!", "max_tokens": 4, "amf_prefix_len": 512}, org_id="org1",
                       tenant_id="t1")
    r3 = w.drain()[0]
    assert r3["amf"]["tier"] == "decode_cache" and r3["output_text"] == r2["output_text"]
    # idempotency
    a = plane.submit({"prompt": "hello", "max_tokens": 2, "idempotency_key": "k"}, org_id="org1")
    assert plane.submit({"prompt": "hello", "max_tokens": 2, "idempotency_key": "k"}, org_id="org1") == a
    w.drain()
    k = plane.kpi_summary("org1")
    assert k["runs"] == 4 and k["hit_rate"] > 0 and k["ttft_hit_ms"]["p50"] is not None
    assert plane.tenant_metrics("t1", "org1")["total_requests"] == 3
    assert plane.billing_report("org1")["tenants"]
    assert plane.restore(j1, "org1")["restored"]
    with pytest.raises(ValueError):
        plane.submit({"prompt": "", "max_tokens": 4})
    with pytest.raises(ValueError):
        plane.submit({"prompt": "x", "max_tokens": 0})


def _req(url, method="GET", body=None, key=None):
    req = urllib.request.Request(url, method=method, data=json.dumps(body).encode() if body is not None else None,
                                 headers={"Content-Type": "application/json"})
    if key:
        req.add_header("Authorization", f"Bearer {key}")
    try:
        with urllib.request.urlopen(req, timeout=30) as r:
            raw = r.read()
            return r.status, (json.loads(raw) if r.headers.get("Content-Type", "").startswith("application/json")
                              else raw.decode())
    except urllib.error.HTTPError as e:
        return e.code, json.loads(e.read() or b"{}")


def test_gateway(tmp_path, monkeypatch):
    from axropus_deploy_b200.cluster.gateway import issue_api_key, serve

    monkeypatch.setenv("KORITH_API_KEY_SALT", "s3cret")
    monkeypatch.setenv("KORITH_RATE_LIMIT_BURST", "1")
    plane, w, _ = _plane(tmp_path)
    key = issue_api_key(plane.ledger, "k1", "org1", rpm=3, tpm=100000)
    httpd = serve(plane, "127.0.0.1", 0, block=False)
    base = f"http://127.0.0.1:{httpd.server_address[1]}"
    try:
        assert _req(base + "/health")[0] == 200
        assert _req(base + "/v1/jobs")[0] == 401
        assert _req(base + "/v1/jobs", key="bad")[0] == 401
        st, out = _req(base + "/v1/jobs", "POST", {"prompt": PROMPT + "hi", "max_tokens": 3}, key)
        assert st == 200 and "job_id" in out
        w.drain()
        st, job = _req(base + f"/v1/jobs/{out['job_id']}", key=key)
        assert st == 200 and job["status"] == "succeeded"
        assert _req(base + f"/v1/jobs/{out['job_id']}/events", key=key)[1]["events"]
        assert _req(base + f"/v1/jobs/{out['job_id']}/metrics", key=key)[1]["lane"] == "MISS"
        assert _req(base + "/v1/snapshots/locations", key=key)[0] == 400
        st, locs = _req(base + f"/v1/snapshots/locations?fingerprint={job['fingerprint_hash']}", key=key)
        assert st == 200 and locs["locations"]
        for p in ("/v1/workers", "/v1/queue_status", "/v1/capabilities", "/v1/cluster/nodes", "/v1/kernels/status",
                  "/v1/kpi/summary", "/v1/alerts", "/v1/metrics/tenant/org1",
                  f"/v1/replay/status?fingerprint={job['fingerprint_hash']}",
                  f"/v1/spec/status?fingerprint={job['fingerprint_hash']}",
                  f"/v1/cluster/routing?fingerprint={job['fingerprint_hash']}"):
            assert _req(base + p, key=key)[0] == 200, p
        assert _req(base + "/v1/billing/report", "POST", {"gpu_hourly_cost": 3.0}, key)[0] == 200
        st, text = _req(base + "/metrics")
        assert st == 200 and "korith_jobs" in text
        assert _req(base + "/v1/jobs", "POST", {"prompt": "x", "max_tokens": 0}, key)[0] == 400
        # rpm 3 with burst 1: the fourth request in this minute is refused
        codes = [_req(base + "/v1/jobs", "POST", {"prompt": "y", "max_tokens": 1}, key)[0] for _ in range(3)]
        assert 429 in codes
        plane.ledger.revoke_api_key("k1", "now")
        assert _req(base + "/v1/jobs", key=key)[0] == 403
    finally:
        httpd.shutdown()
        httpd.server_close()


def test_nodes_and_snapshot_transfer(tmp_path):
    from axropus_deploy_b200.cluster.nodes import NodeRegistry, NodeServer, WorkerRegistry, estimate_transfer_ms

    reg = NodeRegistry()
    reg.register_or_heartbeat("stale", "h", 1, 8, now=time.time() - 100)
    assert [n["node_id"] for n in reg.list_nodes()] == []
    wr = WorkerRegistry()
    wr.register("w0", "n0", 0, "axr_engine")
    assert wr.heartbeat("w0", "busy") and wr.list_workers()[0]["status"] == "busy"
    assert estimate_transfer_ms(10**9, 10.0, 1.0, "ram") == pytest.approx(101.0)

    shared = SqliteLedger(str(tmp_path / "shared.db"))  # one ledger for the cluster
    plane_a, wa, index_a = _plane(tmp_path, "node-a", shared, reg)
    plane_b, wb, _ = _plane(tmp_path, "node-b", shared, reg)
    server = NodeServer("node-a", index_a, registry=reg).start()
    try:
        server.heartbeat_once()
        assert reg.get_node("node-a")["router_port"] == server.port
        plane_a.submit({"prompt": PROMPT + "first", "max_tokens": 3, "amf_prefix_len": 512}, org_id="o")
        ra = wa.drain()[0]
        assert ra["amf"]["decision"] == "miss"
        # node B has never seen the prefix; recomputing is priced high so the snapshot moves
        wb.cold_ms_per_token = 5.0
        plane_b.submit({"prompt": PROMPT + "second", "max_tokens": 3, "amf_prefix_len": 512}, org_id="o")
        rb = wb.drain()[0]
        ev = [json.loads(l) for l in open(tmp_path / "node-b" / "ram" / "o" / rb["job_id"] / "events.jsonl")]
        assert any(e["event"] == "snapshot_transferred" for e in ev), ev
        assert rb["lane"] == "HIT" and rb["amf"]["restored_tokens"] > 0
    finally:
        server.stop()


def test_runtime_governance_and_config(tmp_path):
    from axropus_deploy_b200.cluster.runtime import (DecodeCache, ReplayGovernor, SpecGovernor, SpecKController,
                                                     apply_config_to_env, load_platform_config)

    c = SpecKController()
    assert c.gate({"VERIFY_TOKENS": True}, {})["reason"] == "policy_disabled"
    assert c.gate({}, {"allow_spec": True})["reason"] == "capability_missing"
    for _ in range(3):
        c.update(8, 8, 0.1, 100.0)
    assert c.k == 7 and c.metrics()["decode_ms_saved"] > 0
    for _ in range(20):
        c.update(8, 0)
    assert c.k == SpecKController.MIN_K
    dc = DecodeCache()
    key = dict(org_id="o", backend_id="b", fingerprint_hash="f", prompt_hash="p", sampling_hash="s")
    assert dc.get(**key) is None
    dc.put(**key, output_text="out", tokens_out=3)
    assert dc.get(**key)["output_text"] == "out"
    led = SqliteLedger()
    g = ReplayGovernor(led, negative_roi_max=2, cooldown_ms=1000)
    assert g.record("fp", -1.0)["replay_allowed"]
    assert not g.record("fp", -1.0)["replay_allowed"]
    assert g.status("fp", now=time.time() + 5)["replay_allowed"]
    assert not g.record("fp2", 5.0, corrupted=True)["replay_allowed"]
    sg = SpecGovernor(led, min_accept=0.5, disable_after_n=2)
    assert sg.record("fp", "o", 0.1) and not sg.record("fp", "o", 0.1) and not sg.allowed("fp")
    cfg = tmp_path / "p.yaml"
    cfg.write_text("runtime:\n  spec:\n    k: 6\nsecurity:\n  api_key_salt: abc\n")
    env = {"KORITH_API_KEY_SALT": "keep"}
    set_ = apply_config_to_env(load_platform_config(str(cfg)), env)
    assert set_ == {"KORITH_SPEC_K": "6"} and env["KORITH_API_KEY_SALT"] == "keep"
    with pytest.raises(ValueError):
        apply_config_to_env({"bogus": {}}, {})


def test_dynamo_components():
    from axropus_deploy_b200.cluster.coordinator import AmfCoordinator
    from axropus_deploy_b200.cluster.dynamo import (AmfRouterPlugin, AmfStorageBackend, EventSubscriber,
                                                    KvBlockEvent, prefill_ms, restore_ms)

    # an 8 K Llama-3-8B prefix (1 GiB of bf16 KV) restores faster than it prefills from HBM or
    # host memory, but not from one NVMe drive
    assert restore_ms(8192, "vram") < restore_ms(8192, "ram") < prefill_ms(8192) < restore_ms(8192, "nvme")
    coord = AmfCoordinator()
    coord.register("t", "abc", "n1", "w1", {"tier": "vram"})
    plug = AmfRouterPlugin(coord)
    cands = [{"worker_id": "w0", "node_id": "n0", "kv_overlap": 0.1, "load": 0.2},
             {"worker_id": "w1", "node_id": "n1", "kv_overlap": 0.0, "load": 0.5}]
    best = plug.score_workers(16384, "abc", "t", cands)[0]
    assert best.worker_id == "w1" and best.routed_by == "amf" and best.amf_restore_savings_ms > 0
    assert plug.score_workers(512, "abc", "t", cands)[0].worker_id == "w0"  # short prompt: frontend signals only

    be = AmfStorageBackend(capacity_bytes=0, min_admit_roi=1.5)
    assert not be.register_volume({"capacity_bytes": 0}) and be.register_volume({"capacity_bytes": 1500})
    meta = {"model_hash": "m", "kv_version": 1}
    for i in range(256):  # 256 blocks x 16 tokens = 4096 tokens, 4 bytes each
        be.put(f"a{i}", b"abcd", dict(meta, prefix_id="A", last=i == 255))
    assert be.get("a7", meta) == b"abcd"
    assert be.get("a7", {"model_hash": "other", "kv_version": 1}) is None
    be.put("tiny", b"x", dict(meta, prefix_id="T", last=True))  # 16 tokens: restore not worth it
    assert be.stats()["admission"]["rejected"] == 1
    for i in range(256):
        be.put(f"b{i}", b"efgh", dict(meta, prefix_id="B", last=i == 255))
    st = be.stats()
    assert st["evictions"] == 1 and st["used_bytes"] <= 1500 and be.get("a7") is None and be.get("b3") == b"efgh"
    assert be.delete("b3") and be.get("b3") is None

    kept = []
    sub = EventSubscriber(lambda s: kept.append(s) or True, min_tokens=4096)
    sub.run([KvBlockEvent("created", "w0", "p1", 8192), KvBlockEvent("evicted", "w0", "p1", 8192),
             KvBlockEvent("created", "w0", "p2", 256), KvBlockEvent("evicted", "w0", "p2", 256)])
    assert [k["prefix_hash"] for k in kept] == ["p1"] and sub.stat["skipped"] == 1


def test_codec_ids_and_amf_bench_cli(capsys):
    from axropus_deploy_b200.codecs import AMF_CODEC_FP8, AMF_CODEC_INT4, codec_from_id, codec_id
    from axropus_deploy_b200.server.cli import main

    assert codec_id("int4_g64_asym") == AMF_CODEC_INT4 and codec_from_id(AMF_CODEC_FP8) == "fp8_e4m3"
    with pytest.raises(KeyError):
        codec_id("nvfp4")
    assert main(["amf-bench", "--model", "tiny", "--prompt-tokens", "256", "--max-tokens", "2", "--warm-runs", "1",
                 "--device", "cpu"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out["runs"][0]["tier"] == "cold" and out["runs"][1]["tier"].startswith("g1")


def test_worker_crash_jobs_reclaimed_from_durable_queue(tmp_path):
    """Lane queues on SQLite: a worker that dies holding a job (taken, never acked) loses
    nothing -- a replacement worker over the same queue file picks the job up once the
    visibility timeout has passed, and every submitted job ends succeeded."""
    from axropus_deploy_b200.cluster.adapters import AdapterRegistry
    from axropus_deploy_b200.cluster.control import ControlPlane
    from axropus_deploy_b200.cluster.queues import SqliteQueue
    from axropus_deploy_b200.cluster.worker import ClusterWorker

    ledger = SqliteLedger(str(tmp_path / "ledger.db"))
    qdb = str(tmp_path / "queues.db")
    art = ArtifactStore(tmp_path / "art")
    factory = lambda lane: SqliteQueue(qdb, name=f"w0:{lane}", visibility_s=0.5)  # noqa: E731
    eng = _engine()
    w1 = ClusterWorker("w0", "n0", AdapterRegistry(eng), ledger, art, metrics=MetricsRegistry(), queue_factory=factory)
    plane = ControlPlane(ledger, {"w0": w1}, metrics=w1.metrics)
    ids = [plane.submit({"prompt": f"job {i} " * 8, "max_tokens": 2}, org_id="o") for i in range(3)]
    assert w1.depth() == 3
    assert w1.run_once() is not None                       # one job done and acked
    lane, iid, job = w1._next()                            # the worker takes a second job ...
    assert job["job_id"] in ids
    del w1                                                 # ... and dies without acking it
    w2 = ClusterWorker("w0", "n0", AdapterRegistry(eng), ledger, art, metrics=MetricsRegistry(), queue_factory=factory)
    assert w2.depth() == 1                                 # the abandoned job is in flight, not ready
    time.sleep(0.7)                                        # past the visibility timeout
    done = w2.drain()
    assert len(done) == 2 and all(r["exit_code"] == 0 for r in done)
    assert [ledger.get_job(j)["status"] for j in ids] == ["succeeded"] * 3
    assert w2.depth() == 0


def test_more_adapters_and_proxy(tmp_path):
    """vLLM-style adapter request extras and the in-process transformers adapter, against a
    stub OpenAI server; the reverse proxy routes a prompt to the worker that holds its prefix."""
    import threading
    from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

    from axropus_deploy_b200.amf.keys import pool_key
    from axropus_deploy_b200.cluster.adapters import AdapterRegistry, TransformersAdapter, VllmOpenAIAdapter
    from axropus_deploy_b200.cluster.coordinator import AmfCoordinator
    from axropus_deploy_b200.cluster.gateway import serve_proxy
    from axropus_deploy_b200.cluster.router import ClusterRouter, WorkerInfo

    seen = []

    def stub(name):
        class H(BaseHTTPRequestHandler):
            def log_message(self, *a):
                pass

            def do_POST(self):
                body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
                seen.append((name, body))
                out = json.dumps({"choices": [{"text": "ok"}], "token_ids": [111, 107], "server": name,
                                  "usage": {"kv_transfer_params": {"blk": 3}, "accepted_speculative_tokens": 3,
                                            "proposed_speculative_tokens": 4},
                                  "axropus": {"hit": True, "tier": "g1_raw", "ttft_ms": 1.5}}).encode()
                self.send_response(200)
                self.send_header("Content-Type", "application/json")
                self.send_header("Content-Length", str(len(out)))
                self.end_headers()
                self.wfile.write(out)
        srv = ThreadingHTTPServer(("127.0.0.1", 0), H)
        threading.Thread(target=srv.serve_forever, daemon=True).start()
        return srv

    a, b = stub("a"), stub("b")
    try:
        url_a, url_b = (f"http://127.0.0.1:{s.server_address[1]}" for s in (a, b))
        v = VllmOpenAIAdapter(url_a, "m")
        r = v.run_speculative("hello", 4, {"temperature": 0}, {"lane": "SPEC_HIT", "priority": 2}, {}, None,
                              spec_cfg={"k": 4})
        body = seen[-1][1]
        assert body["num_speculative_tokens"] == 4 and body["vllm_xargs"]["korith_lane"] == "SPEC_HIT"
        assert r["kv_transfer_params"] == {"blk": 3} and r["spec"]["accepted"] == 3 and r["amf"]["decision"] == "hit"
        assert AdapterRegistry().get_adapter({"backend_id": "vllm_openai", "model": {"endpoint": url_a}}).backend_id \
            == "vllm_openai"
        hf = TransformersAdapter()
        out = hf.run_baseline("abc", 3, {}, {}, {}, None)
        assert out["tokens_out"] == 3
        ver = hf.verify_tokens("abc", out["output_tokens"], {})
        assert ver["accepted"] == 3  # the model's own greedy tokens verify in full
        # proxy: the coordinator says worker "b" holds this prompt's prefix
        text = "x" * 600
        coord = AmfCoordinator()
        coord.register("default", pool_key(list(text.encode())[:512]), "nb", "b", {})
        router = ClusterRouter([WorkerInfo("a", "na"), WorkerInfo("b", "nb")], coordinator=coord, prefix_tokens=512)
        px = serve_proxy({"a": url_a, "b": url_b}, router)
        try:
            purl = f"http://127.0.0.1:{px.server_address[1]}/v1/completions"
            req = urllib.request.Request(purl, data=json.dumps({"prompt": text, "max_tokens": 4}).encode(),
                                         method="POST", headers={"Content-Type": "application/json"})
            with urllib.request.urlopen(req, timeout=30) as resp:
                assert json.loads(resp.read())["server"] == "b"
                assert resp.headers["X-Korith-Route"] == "amf_local:b"
            assert router.workers["b"].load == 0
        finally:
            px.shutdown()
            px.server_close()
    finally:
        for s in (a, b):
            s.shutdown()
            s.server_close()


def test_snapshot_sidecar_validation(tmp_path):
    """The .meta.json sidecar refuses a snapshot for another model, tokenizer, layout,
    context size or fingerprint, and a snapshot whose bytes changed."""
    from axropus_deploy_b200.cluster.engine_client import validate_snapshot_metadata, write_snapshot_metadata

    snap = tmp_path / "s.amfk"
    snap.write_bytes(bytes(range(256)) * 64)
    ctx = dict(fingerprint_hash="fp", model_hash="m", tokenizer_hash="t", kv_layout_version="paged16", n_ctx=4096)
    write_snapshot_metadata(snap, backend_id="axr_engine", created_at="now", **ctx)
    assert validate_snapshot_metadata(snap, **ctx)[:2] == (True, "ok")
    for k, v, reason in (("model_hash", "m2", "snapshot_model_mismatch"), ("tokenizer_hash", "t2", "snapshot_tokenizer_mismatch"),
                         ("kv_layout_version", "x", "snapshot_layout_mismatch"), ("n_ctx", 8192, "snapshot_ctx_mismatch"),
                         ("fingerprint_hash", "other", "snapshot_fingerprint_mismatch")):
        assert validate_snapshot_metadata(snap, **dict(ctx, **{k: v}))[1] == reason
    raw = bytearray(snap.read_bytes())
    raw[100] ^= 1
    snap.write_bytes(bytes(raw))
    assert validate_snapshot_metadata(snap, **ctx)[1] == "snapshot_checksum_mismatch"
    assert validate_snapshot_metadata(tmp_path / "missing.amfk", **ctx)[1] == "snapshot_missing"


def test_concurrent_worker_batches_jobs(tmp_path):
    """A worker with several jobs in flight over one EngineService: the engine runs them in
    the same steps (continuous batching) and every job succeeds."""
    from axropus_deploy_b200.cluster.adapters import AdapterRegistry
    from axropus_deploy_b200.cluster.control import ControlPlane
    from axropus_deploy_b200.cluster.worker import ClusterWorker
    from axropus_deploy_b200.server.service import EngineService

    eng = _engine()
    peak = {"running": 0}
    step = eng.step

    def counting_step():
        peak["running"] = max(peak["running"], len(eng.running) + len(eng.waiting))
        return step()

    eng.step = counting_step
    svc = EngineService(eng)
    ledger = SqliteLedger(str(tmp_path / "l.db"))
    w = ClusterWorker("w0", "n0", AdapterRegistry(eng, service=svc), ledger, ArtifactStore(tmp_path / "art"),
                      metrics=MetricsRegistry(), concurrency=4)
    plane = ControlPlane(ledger, {"w0": w}, metrics=w.metrics)
    ids = [plane.submit({"prompt": f"request {i} " * 6, "max_tokens": 8}, org_id="o") for i in range(6)]
    w.start()
    try:
        deadline = time.time() + 120
        while time.time() < deadline and any(ledger.get_job(j)["status"] != "succeeded" for j in ids):
            time.sleep(0.05)
    finally:
        w.stop()
        svc._stop.set()
    assert [ledger.get_job(j)["status"] for j in ids] == ["succeeded"] * 6
    assert peak["running"] >= 2  # jobs shared engine steps
