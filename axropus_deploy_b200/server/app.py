"""OpenAI-compatible HTTP server over the AMF-backed engine.

Endpoints as in the reference (axropus/server.py:121-189): ``/healthz``, ``/metrics``
(Prometheus), ``/stats``, ``/v1/chat/completions``, ``/v1/completions``, optional
bearer key. Unlike the reference -- which runs a plain ``LLM.generate`` and stores a
zero-filled stub KV on a miss (server.py:217-242) -- requests here run through the
engine: a hit restores the prefix KV into the live cache and prefills only the
suffix, a miss prefills and captures. Token ids can be sent directly
(``prompt_token_ids``). When ``AXROPUS_MODEL`` names a Hugging Face model directory the
engine serves its weights (``models/loader.py``) and text goes through its
``tokenizer.json`` (``models/tokenizer.py``), with the Llama-3 chat template for chat
requests; without one, text falls back to byte-level tokens like the reference.
"""
from __future__ import annotations

import asyncio
import logging
import time
from typing import Any, Dict, List, Optional

from fastapi import FastAPI, Header, HTTPException, Request
from fastapi.responses import Response

from ..amf.prompt_policy import prepare_prompt
from ..config import AxropusConfig, KorithConfig
from ..engine import SamplingParams
from .metrics import MetricRegistry
from .service import EngineService

log = logging.getLogger(__name__)


def render_messages(messages: List[Dict[str, Any]], tokenizer=None) -> str:
    if tokenizer is not None and "<|start_header_id|>" in tokenizer.added:
        # Llama-3 chat format: header per turn, end-of-turn marks, assistant header last
        out = "<|begin_of_text|>"
        for m in messages:
            out += f"<|start_header_id|>{m.get('role', 'user')}<|end_header_id|>\n\n{m.get('content', '')}<|eot_id|>"
        return out + "<|start_header_id|>assistant<|end_header_id|>\n\n"
    return "".join(f"<|{m.get('role', 'user')}|>{m.get('content', '')}<|/{m.get('role', 'user')}|>" for m in messages)


def byte_tokens(text: str) -> List[int]:
    return list(text.encode("utf-8", "replace"))


def detok(tokens: List[int]) -> str:
    return bytes(t % 256 for t in tokens).decode("utf-8", "replace")


def load_tokenizer(model_dir: str):
    """The model directory's tokenizer.json, or None."""
    import os

    from ..models.tokenizer import Tokenizer

    p = os.path.join(model_dir, "tokenizer.json")
    return Tokenizer.from_file(p) if os.path.isfile(p) else None


def is_model_dir(path: str) -> bool:
    import os

    return bool(path) and os.path.isfile(os.path.join(path, "config.json"))


def build_engine(cfg: AxropusConfig, kcfg: Optional[KorithConfig] = None, *, num_blocks: Optional[int] = None):
    """Engine + AMF tiers from the AXROPUS_* / KORITH_* configuration."""
    import torch

    from ..amf import AmfManager, DiskTier, G1Pool, LMCacheAdapter
    from ..amf.keys import AmfContext, amf_float_bits, amf_hash_model_name, amf_hash_tenant_id
    from ..engine import EngineConfig, LLMEngine
    from ..models.config import PRESETS, get_config
    from ..models.llama import LlamaModel
    from ..amf.pool import PoolSlab

    kcfg = kcfg or KorithConfig.from_env()
    dev = torch.device(cfg.device if (cfg.device == "cpu" or torch.cuda.is_available()) else "cpu")
    if is_model_dir(cfg.model):  # a Hugging Face checkpoint directory
        from ..models.loader import load_pretrained

        model = load_pretrained(cfg.model, dev)
        mc = model.cfg
    else:
        name = cfg.model if cfg.model in PRESETS else "tiny128"
        mc = get_config(name)
        model = LlamaModel(mc, dev, seed=0)
    amf = None
    if kcfg.enable_amf or kcfg.vram_cache_gb or kcfg.vram_pool_gb:
        raw = comp = None
        if kcfg.vram_cache_gb > 0:
            chunk = PoolSlab.chunk_bytes(mc.num_layers, mc.num_kv_heads, mc.head_dim, "raw")
            raw = G1Pool(mc.num_layers, mc.num_kv_heads, mc.head_dim, "raw",
                         max(1, int(kcfg.vram_cache_gb * (1 << 30) // chunk)), dev)
        if kcfg.vram_pool_gb > 0:
            chunk = PoolSlab.chunk_bytes(mc.num_layers, mc.num_kv_heads, mc.head_dim, kcfg.vram_pool_quant)
            comp = G1Pool(mc.num_layers, mc.num_kv_heads, mc.head_dim, kcfg.vram_pool_quant,
                          max(1, int(kcfg.vram_pool_gb * (1 << 30) // chunk)), dev)
        if raw is None and comp is None:
            raw = G1Pool(mc.num_layers, mc.num_kv_heads, mc.head_dim, "raw", 256, dev)
        tenant_hash = amf_hash_tenant_id(kcfg.tenant_id) if kcfg.amf_tenant_isolation else 0
        ctx = AmfContext(model_hash=amf_hash_model_name(mc.name), tenant_hash=tenant_hash,
                         n_ctx=kcfg.n_ctx, kv_version=1, rope_base_bits=amf_float_bits(mc.rope_theta),
                         rope_scale_bits=amf_float_bits(1.0))
        disk = DiskTier(kcfg.amf_path, ctx, from_env=True) if kcfg.enable_amf else None
        lm = LMCacheAdapter(enabled=cfg.lmcache_enabled or kcfg.lmcache_fallback, backend=cfg.lmcache_backend,
                            path=cfg.lmcache_path, lookup_timeout_ms=kcfg.lmcache_lookup_timeout_ms)
        amf = AmfManager(raw_pool=raw, comp_pool=comp, lmcache=lm, disk=disk, min_tokens=kcfg.amf_min_tokens,
                         vram_first=kcfg.amf_vram_first, sync_save=kcfg.amf_sync_save,
                         lmcache_fallback=kcfg.lmcache_fallback, promote_lmcache_hits=kcfg.promote_lmcache_hits,
                         lmcache_write_through=kcfg.lmcache_write_through, write_policy=cfg.write_policy,
                         large_write_threshold=cfg.large_write_threshold, disable_restore=kcfg.amf_disable_restore)
    ecfg = EngineConfig(num_blocks=num_blocks or (4096 if dev.type == "cuda" else 512), kv_fmt=kcfg.kv_cache_dtype,
                        max_batch=kcfg.n_seq_max, max_model_len=min(kcfg.n_ctx, mc.max_position),
                        amf_min_tokens=kcfg.amf_min_tokens, cuda_graphs=kcfg.cuda_graphs and dev.type == "cuda")
    return LLMEngine(model, ecfg, amf)


def create_app(cfg: AxropusConfig, engine=None, tokenizer=None):
    eng = engine or build_engine(cfg)
    tok = tokenizer if tokenizer is not None else (load_tokenizer(cfg.model) if is_model_dir(cfg.model) else None)
    encode = (lambda text: tok.encode(text)) if tok is not None else byte_tokens
    decode = tok.decode if tok is not None else detok
    svc = EngineService(eng)
    metrics = MetricRegistry(cfg.enable_prometheus)
    from contextlib import asynccontextmanager

    @asynccontextmanager
    async def lifespan(_app):
        yield
        svc.close()

    app = FastAPI(title="axropus_deploy_b200", version="0.1.0", lifespan=lifespan)
    app.state.service = svc

    def check(auth: Optional[str]) -> None:
        if not cfg.api_key:
            return
        if not auth or not auth.startswith("Bearer ") or auth.split(" ", 1)[1] != cfg.api_key:
            raise HTTPException(status_code=401, detail="missing or bad bearer token")

    @app.get("/healthz")
    def healthz():
        return {"ok": True, "model": eng.model.cfg.name, "device": str(eng.device), "amf": eng.amf is not None,
                "tokenizer": "tokenizer.json" if tok is not None else "bytes"}

    @app.get("/metrics")
    def prom():
        if eng.amf is not None and eng.amf.target_pool() is not None:
            metrics.update_pool(eng.amf.target_pool().stats())
        return Response(content=metrics.render(), media_type="text/plain; version=0.0.4")

    @app.get("/stats")
    def stats():
        return eng.stats()

    async def run(body: Dict[str, Any], prompt_ids: List[int]) -> Dict[str, Any]:
        t0 = time.perf_counter()
        params = SamplingParams(max_tokens=int(body.get("max_tokens", 16)),
                                temperature=float(body.get("temperature", 0.0)), seed=body.get("seed"))
        fut = svc.submit(prompt_ids, params, body.get("amf_prefix_len"))
        r = await asyncio.wrap_future(fut)
        lat = (time.perf_counter() - t0) * 1e3
        metrics.observe_request(r.amf_tier, r.ttft_ms, r.restored_tokens)
        from ..amf.keys import pool_key

        return {
            "id": f"cmpl-{r.req_id}", "created": int(time.time()), "model": eng.model.cfg.name,
            "usage": {"prompt_tokens": len(prompt_ids), "completion_tokens": len(r.output),
                      "total_tokens": len(prompt_ids) + len(r.output)},
            "token_ids": r.output, "text": decode(r.output),
            "axropus": {"tier": r.amf_tier, "hit": r.amf_tier != "cold", "latency_ms": round(lat, 3),
                        "ttft_ms": round(r.ttft_ms, 3), "restored_tokens": r.restored_tokens,
                        "prefix_hash": pool_key(prompt_ids[: (len(prompt_ids) - 1) // 16 * 16])},
        }

    @app.post("/v1/completions")
    async def completions(request: Request, authorization: Optional[str] = Header(default=None)):
        check(authorization)
        body = await request.json()
        ids = body.get("prompt_token_ids")
        if ids is None:
            p = body.get("prompt", "")
            if isinstance(p, list):
                ids = p
            else:  # canonical text, and the AMF prefix it keys on (KORITH_AMF_* prompt policy)
                prep = prepare_prompt(str(p), encode)
                ids = prep["tokens"]
                if body.get("amf_prefix_len") is None and prep["amf_prefix_len"] is not None:
                    body["amf_prefix_len"] = prep["amf_prefix_len"]
        out = await run(body, [int(x) for x in ids])
        metrics.requests.labels(endpoint="completions").inc()
        out.update(object="text_completion",
                   choices=[{"index": 0, "text": out.pop("text"), "finish_reason": "length"}])
        return out

    @app.post("/v1/chat/completions")
    async def chat(request: Request, authorization: Optional[str] = Header(default=None)):
        check(authorization)
        body = await request.json()
        ids = body.get("prompt_token_ids")
        if not ids:
            prep = prepare_prompt(render_messages(body.get("messages") or [], tok), encode)
            ids = prep["tokens"]
            if body.get("amf_prefix_len") is None and prep["amf_prefix_len"] is not None:
                body["amf_prefix_len"] = prep["amf_prefix_len"]
        out = await run(body, [int(x) for x in ids])
        metrics.requests.labels(endpoint="chat").inc()
        out.update(object="chat.completion",
                   choices=[{"index": 0, "message": {"role": "assistant", "content": out.pop("text")},
                             "finish_reason": "length"}])
        return out

    return app
