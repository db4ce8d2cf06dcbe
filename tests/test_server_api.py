"""Serving layer on CPU: HTTP endpoints with real KV reuse, bearer auth, Prometheus
names, the amf_save_kv / amf_restore_kv worker API, the CLI and the config surface."""
import json

import numpy as np
import pytest
import torch

from axropus_deploy_b200.config import AxropusConfig, KorithConfig


@pytest.fixture(scope="module")
def client():
    from fastapi.testclient import TestClient

    from axropus_deploy_b200.server.app import build_engine, create_app

    cfg = AxropusConfig(model="tiny", device="cpu", api_key="sekret")
    k = KorithConfig()
    k.enable_amf = False
    k.vram_cache_gb = 0.05
    k.n_ctx = 2048
    k.n_seq_max = 8
    eng = build_engine(cfg, k, num_blocks=256)
    with TestClient(create_app(cfg, eng)) as c:
        c.engine = eng
        yield c


def test_auth_and_health(client):
    assert client.get("/healthz").json()["ok"]
    assert client.post("/v1/completions", json={"prompt": "hi"}).status_code == 401


def test_completions_hit_after_cold(client):
    h = {"Authorization": "Bearer sekret"}
    g = torch.Generator().manual_seed(3)
    prefix = torch.randint(0, 32000, (256,), generator=g).tolist()
    r1 = client.post("/v1/completions", headers=h,
                     json={"prompt_token_ids": prefix + [1, 2, 3], "max_tokens": 4, "amf_prefix_len": 256}).json()
    assert r1["axropus"]["tier"] == "cold" and len(r1["token_ids"]) == 4
    client.engine.evict_live_cache()
    r2 = client.post("/v1/completions", headers=h,
                     json={"prompt_token_ids": prefix + [1, 2, 3], "max_tokens": 4, "amf_prefix_len": 256}).json()
    assert r2["axropus"]["tier"] == "g1_raw" and r2["axropus"]["restored_tokens"] == 256
    assert r2["token_ids"] == r1["token_ids"]
    r3 = client.post("/v1/chat/completions", headers=h,
                     json={"messages": [{"role": "user", "content": "hello there"}], "max_tokens": 2}).json()
    assert r3["object"] == "chat.completion" and r3["usage"]["completion_tokens"] == 2
    text = client.get("/metrics").text
    for name in ("axropus_cache_hits_total", "axropus_pool_prefixes_resident", "axropus_tokens_saved_total",
                 "axropus_pool_bytes_used"):
        assert name in text
    st = client.get("/stats").json()
    assert st["amf"]["hits_g1_raw"] >= 1


def test_worker_api(client):
    from axropus_deploy_b200.amf.worker_api import AmfWorkerExtension

    svc = client.app.state.service
    g = torch.Generator().manual_seed(4)
    toks = torch.randint(0, 32000, (160,), generator=g).tolist()
    svc.submit(toks + [5]).result(timeout=60)

    def worker_calls(eng):
        w = AmfWorkerExtension(eng)
        saved = w.call("amf_save_kv", toks)  # blocks found through the prefix cache
        blocks = eng.bm.allocate(10)
        try:
            return saved, w.amf_restore_kv(toks, blocks), w.amf_restore_kv(list(range(160)), blocks)
        finally:
            eng.bm.release(blocks)

    saved, hit, miss = svc.run_in_engine(worker_calls).result(timeout=60)
    assert saved and hit == 160 and miss == 0


def test_config_surface(monkeypatch, tmp_path):
    monkeypatch.setenv("AXROPUS_PORT", "9001")
    monkeypatch.setenv("AXROPUS_LMCACHE_ENABLE", "yes")
    monkeypatch.setenv("KORITH_VRAM_POOL_GB", "8")
    monkeypatch.setenv("KORITH_VRAM_POOL_QUANT", "int4")
    monkeypatch.setenv("KORITH_KV_FP8", "1")
    monkeypatch.setenv("KORITH_AMF_MIN_TOKENS", "oops")
    monkeypatch.setenv("KORITH_CUDA_GRAPH_CACHE_SIZE", "999")
    a = AxropusConfig.from_env()
    assert a.port == 9001 and a.lmcache_enabled
    k = KorithConfig.from_env()
    assert k.vram_pool_gb == 8.0 and k.vram_pool_quant == "int4" and k.kv_cache_dtype == "fp8"
    assert k.amf_min_tokens == 64 and k.cuda_graph_cache_size == 64
    f = tmp_path / "c.yaml"
    f.write_text("port: 7000\nmodel: llama3-8b\nwrite_policy: always\n")
    c = AxropusConfig.load(f, {"host": "127.0.0.1"})
    assert c.port == 9001 and c.model == "llama3-8b" and c.write_policy == "always" and c.host == "127.0.0.1"
    assert "api_key" not in c.summary()


def test_cli_bench_quick(capsys):
    from axropus_deploy_b200.server.cli import main

    assert main(["bench", "--quick"]) == 0
    out = json.loads(capsys.readouterr().out)
    assert out["codec_sweep"]["fp8_e4m3"]["rel_err"] < 0.05
