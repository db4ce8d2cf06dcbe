"""Configuration surface: ``AXROPUS_*`` server config and the ``KORITH_*`` knobs.

Two objects:

* :class:`AxropusConfig` -- the serving config (model, HTTP, pool shape, router
  policy, LMCache tier, telemetry). Same field names, defaults and ``AXROPUS_*``
  variables as the reference (axropus/config.py:47-162), composed env -> YAML file
  -> explicit overrides.
* :class:`KorithConfig` -- every ``KORITH_*`` variable the reference's engine,
  store, scheduler and README define (engine.cpp:344-393, :553-589, :2161-2275;
  amf_store.cpp:307-423; decode_scheduler.py:89-147; README.md:41-131). The
  README-only knobs (``KORITH_VRAM_CACHE_GB``, ``KORITH_VRAM_POOL_GB``,
  ``KORITH_VRAM_POOL_QUANT``, ``KORITH_AMF_VRAM_FIRST``, ``KORITH_AMF_SYNC_SAVE``,
  ``KORITH_VRAM_CACHE_DEVICE``, ``AXROPUS_LMCACHE_*``) have no reader in the
  reference; their meaning here follows the README's description.

Parsing rules follow the reference's C++ parsers: integers must parse completely,
booleans accept 1/true/yes/on and 0/false/no/off, anything else keeps the default.
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field, fields
from pathlib import Path
from typing import Any, Dict, Optional

_TRUE = {"1", "true", "TRUE", "True", "yes", "on"}
_FALSE = {"0", "false", "FALSE", "False", "no", "off"}


def env_bool(name: str, default: bool) -> bool:
    v = os.environ.get(name)
    if v is None or v == "":
        return default
    if v in _TRUE:
        return True
    if v in _FALSE:
        return False
    return default


def env_int(name: str, default: int, minimum: Optional[int] = None) -> int:
    v = os.environ.get(name)
    if v is None or v == "":
        return default
    try:
        x = int(v, 10)
    except ValueError:
        return default
    if minimum is not None and x < minimum:
        return default
    return x


def env_float(name: str, default: float, lo: Optional[float] = None, hi: Optional[float] = None) -> float:
    v = os.environ.get(name)
    if v is None or v == "":
        return default
    try:
        x = float(v)
    except ValueError:
        return default
    if x != x or x in (float("inf"), float("-inf")):
        return default
    if lo is not None and x < lo:
        return default
    if hi is not None and x > hi:
        return default
    return x


def env_str(name: str, default: str) -> str:
    v = os.environ.get(name)
    return default if v is None else v


# --------------------------------------------------------------------------------------
# AXROPUS_* serving config
# --------------------------------------------------------------------------------------
@dataclass
class AxropusConfig:
    """Runtime configuration for the AMF server, router and pool."""

    model: str = "meta-llama/Llama-3.1-70B"
    tenant_id: str = "__shared__"
    host: str = "0.0.0.0"
    port: int = 8001
    metrics_port: int = 9090
    api_key: str = ""
    num_layers: int = 80
    num_kv_heads: int = 8
    head_dim: int = 128
    bytes_per_layer: int = 1 << 30
    block_bytes: int = 1 << 17
    default_format: str = "int4_sym_block"
    device: str = "cuda"
    min_prefix_tokens: int = 64
    write_policy: str = "large_only"
    large_write_threshold: int = 2048
    lmcache_enabled: bool = False
    lmcache_backend: str = "cpu"
    lmcache_path: str = "/tmp/axropus_lmcache"
    lmcache_url: str = ""
    disable_cuda_build: bool = False
    enable_prometheus: bool = True
    log_level: str = "INFO"

    _ENV = {
        "model": "AXROPUS_MODEL",
        "tenant_id": "AXROPUS_TENANT_ID",
        "host": "AXROPUS_HOST",
        "port": "AXROPUS_PORT",
        "metrics_port": "AXROPUS_METRICS_PORT",
        "api_key": "AXROPUS_API_KEY",
        "num_layers": "AXROPUS_NUM_LAYERS",
        "num_kv_heads": "AXROPUS_NUM_KV_HEADS",
        "head_dim": "AXROPUS_HEAD_DIM",
        "bytes_per_layer": "AXROPUS_BYTES_PER_LAYER",
        "block_bytes": "AXROPUS_BLOCK_BYTES",
        "default_format": "AXROPUS_DEFAULT_FORMAT",
        "device": "AXROPUS_DEVICE",
        "min_prefix_tokens": "AXROPUS_MIN_PREFIX_TOKENS",
        "write_policy": "AXROPUS_WRITE_POLICY",
        "large_write_threshold": "AXROPUS_LARGE_WRITE_THRESHOLD",
        "lmcache_enabled": "AXROPUS_LMCACHE_ENABLE",
        "lmcache_backend": "AXROPUS_LMCACHE_BACKEND",
        "lmcache_path": "AXROPUS_LMCACHE_PATH",
        "lmcache_url": "AXROPUS_LMCACHE_URL",
        "disable_cuda_build": "AXROPUS_DISABLE_CUDA_BUILD",
        "enable_prometheus": "AXROPUS_ENABLE_PROMETHEUS",
        "log_level": "AXROPUS_LOG_LEVEL",
    }

    @classmethod
    def from_env(cls) -> "AxropusConfig":
        cfg = cls()
        for f in fields(cls):
            name = cls._ENV.get(f.name)
            if name is None:
                continue
            cur = getattr(cfg, f.name)
            if isinstance(cur, bool):
                setattr(cfg, f.name, env_bool(name, cur))
            elif isinstance(cur, int):
                setattr(cfg, f.name, env_int(name, cur))
            else:
                setattr(cfg, f.name, env_str(name, cur))
        return cfg

    @classmethod
    def from_yaml(cls, path: str | Path) -> "AxropusConfig":
        text = Path(path).read_text()
        try:
            import yaml

            data = yaml.safe_load(text) or {}
        except ImportError:  # pragma: no cover - yaml is installed here
            data = json.loads(text)
        names = {f.name for f in fields(cls)}
        return cls(**{k: v for k, v in data.items() if k in names})

    @classmethod
    def load(cls, config_file: Optional[str | Path] = None,
             overrides: Optional[Dict[str, Any]] = None) -> "AxropusConfig":
        """defaults -> YAML file -> AXROPUS_* env (non-default wins) -> overrides."""
        cfg = cls.from_env()
        if config_file:
            file_cfg = cls.from_yaml(config_file)
            for f in fields(cls):
                if getattr(cfg, f.name) == f.default:
                    setattr(cfg, f.name, getattr(file_cfg, f.name))
        for k, v in (overrides or {}).items():
            if v is not None and hasattr(cfg, k):
                setattr(cfg, k, v)
        return cfg

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)

    def summary(self) -> str:
        d = self.to_dict()
        d.pop("api_key", None)
        return "\n".join(f"  {k}: {v}" for k, v in sorted(d.items()))


# --------------------------------------------------------------------------------------
# KORITH_* knobs
# --------------------------------------------------------------------------------------
@dataclass
class KorithConfig:
    # master / paths
    enable_amf: bool = False
    amf_path: str = "amf"
    amf_min_tokens: int = 64
    tenant_id: str = "__shared__"
    # disk store budget / eviction (consumed natively by the AmfStore; mirrored here)
    amf_max_bytes: int = 512 << 20
    amf_storage_budget_gb: float = 0.0
    amf_eviction_watermark: float = 0.90
    amf_eviction_policy: str = "lru"
    amf_hot_ttl_s: int = 300
    amf_warm_ttl_s: int = 3600
    amf_default_ttl_s: int = 86400
    amf_max_ttl_s: int = 604800
    amf_max_age_ms: int = 0
    # ROI
    amf_min_prompt_ms: float = 0.0
    amf_min_roi: float = 0.0
    amf_min_admit_roi: float = 0.0
    amf_low_roi_hits: int = 3
    # integrity / prewarm / disk
    amf_model_version_check: bool = True
    amf_prewarm: bool = False
    amf_prewarm_top_k: int = 10
    amf_prewarm_timeout_s: int = 30
    amf_disk_guard: bool = True
    amf_min_free_disk_bytes: int = 0
    amf_min_free_disk_pct: float = 0.0
    # engine AMF behaviour
    amf_direct_gpu: bool = True
    amf_disable_restore: bool = False
    amf_shared_prefixes: bool = False
    amf_shared_prefix_patterns: str = ""
    amf_prefix_extraction: bool = False
    amf_prefix_boundary_token: str = "<|user|>"
    amf_tenant_isolation: bool = False  # off: one key namespace (tenant hash 0), as the reference's store
    amf_normalize_whitespace: bool = False
    amf_normalize_unicode: bool = False
    amf_prompt_collapse_blanks: bool = False
    amf_prompt_strip_outer: bool = False
    amf_canonicalize_template_json: bool = False
    # README-defined G1 tiers
    amf_vram_first: bool = True
    amf_sync_save: bool = False
    vram_cache_device: str = "cuda"
    vram_cache_gb: float = 0.0
    vram_pool_gb: float = 0.0
    vram_pool_quant: str = "fp8"
    lmcache_fallback: bool = False
    promote_lmcache_hits: bool = True
    lmcache_write_through: bool = False
    lmcache_lookup_timeout_ms: int = 50
    # KV / model / GPU
    kv_fp8: bool = False
    kv_type_k: str = ""
    kv_type_v: str = ""
    tensor_split: str = ""
    main_gpu: int = 0
    n_ctx: int = 8192
    n_batch: int = 512
    n_seq_max: int = 64
    allow_n_ctx_fallback: bool = True
    cuda_graphs: bool = True
    cuda_graph_cache_size: int = 4
    cuda_graph_capture: bool = False
    batch_tokens: int = 256
    # spec decode
    draft_model: str = ""
    spec_v2: bool = False
    spec_v3: bool = False
    spec_depth: int = 0
    spec_k: int = 4
    spec_min_accept: float = 0.0
    spec_allow_exec: bool = True
    spec_allow_commit: bool = True
    spec_pause: bool = False
    max_depth: int = 16
    scheduler_lib: str = ""
    # vLLM-style scheduler knobs (decode-first reordering)
    sched_decode_first: bool = True
    sched_adaptive_budget: bool = True
    sched_budget_scale_decode: float = 1.0
    sched_decode_ratio_threshold: float = 0.5
    sched_min_scheduled_tokens: int = 1
    sched_starvation_s: float = 2.0
    sched_prefill_penalty: float = 0.0
    sched_short_decode_bonus: float = 0.0
    sched_decode_full_budget_on_hit: bool = True
    sched_trace_path: str = ""
    sched_trace_every: int = 0
    # observability
    engine_events_path: str = ""
    engine_metrics_path: str = ""
    mf_snapshot_in: str = ""
    mf_snapshot_out: str = ""

    @classmethod
    def from_env(cls) -> "KorithConfig":
        c = cls()
        e = c
        e.enable_amf = (os.environ.get("KORITH_ENABLE_AMF", "") or "0")[0] != "0"
        e.amf_path = os.environ.get("KORITH_AMF_PATH") or "amf"
        e.amf_min_tokens = env_int("KORITH_AMF_MIN_TOKENS", e.amf_min_tokens, minimum=1)
        e.tenant_id = env_str("KORITH_TENANT_ID", e.tenant_id) or "__shared__"
        e.amf_max_bytes = env_int("KORITH_AMF_MAX_BYTES", e.amf_max_bytes, minimum=1)
        e.amf_storage_budget_gb = env_float("KORITH_AMF_STORAGE_BUDGET_GB", 0.0, lo=0.0)
        e.amf_eviction_watermark = env_float("KORITH_AMF_EVICTION_WATERMARK", e.amf_eviction_watermark, 1e-9, 1.0)
        pol = os.environ.get("KORITH_AMF_EVICTION_POLICY", "")
        if pol in ("lru", "lfu", "roi"):
            e.amf_eviction_policy = pol
        e.amf_hot_ttl_s = env_int("KORITH_AMF_HOT_TTL_S", e.amf_hot_ttl_s, minimum=1)
        e.amf_warm_ttl_s = env_int("KORITH_AMF_WARM_TTL_S", e.amf_warm_ttl_s, minimum=1)
        e.amf_hot_ttl_s = min(e.amf_hot_ttl_s, e.amf_warm_ttl_s)
        e.amf_default_ttl_s = env_int("KORITH_AMF_DEFAULT_TTL_S", e.amf_default_ttl_s, minimum=1)
        e.amf_max_ttl_s = max(env_int("KORITH_AMF_MAX_TTL_S", e.amf_max_ttl_s, minimum=1), e.amf_default_ttl_s)
        e.amf_max_age_ms = env_int("KORITH_AMF_MAX_AGE_MS", e.amf_max_age_ms, minimum=0)
        e.amf_min_prompt_ms = env_float("KORITH_AMF_MIN_PROMPT_MS", 0.0, lo=0.0)
        e.amf_min_roi = env_float("KORITH_AMF_MIN_ROI", 0.0, lo=0.0)
        e.amf_min_admit_roi = env_float("KORITH_AMF_MIN_ADMIT_ROI", 0.0, lo=0.0)
        e.amf_low_roi_hits = env_int("KORITH_AMF_LOW_ROI_HITS", e.amf_low_roi_hits, minimum=1)
        e.amf_model_version_check = env_bool("KORITH_AMF_MODEL_VERSION_CHECK", True)
        e.amf_prewarm = env_bool("KORITH_AMF_PREWARM", False)
        e.amf_prewarm_top_k = env_int("KORITH_AMF_PREWARM_TOP_K", e.amf_prewarm_top_k, minimum=1)
        e.amf_prewarm_timeout_s = env_int("KORITH_AMF_PREWARM_TIMEOUT_S", e.amf_prewarm_timeout_s, minimum=0)
        e.amf_disk_guard = env_bool("KORITH_AMF_DISK_GUARD", True)
        e.amf_min_free_disk_bytes = env_int("KORITH_AMF_MIN_FREE_DISK_BYTES", 0, minimum=0)
        e.amf_min_free_disk_pct = env_float("KORITH_AMF_MIN_FREE_DISK_PCT", 0.0, 0.0, 1.0)
        e.amf_direct_gpu = env_bool("KORITH_AMF_DIRECT_GPU", e.amf_direct_gpu)
        e.amf_disable_restore = env_bool("KORITH_AMF_DISABLE_RESTORE", False)
        e.amf_shared_prefixes = env_bool("KORITH_AMF_SHARED_PREFIXES", False)
        e.amf_shared_prefix_patterns = env_str("KORITH_AMF_SHARED_PREFIX_PATTERNS", "")
        e.amf_prefix_extraction = env_bool("KORITH_AMF_PREFIX_EXTRACTION", False)
        e.amf_prefix_boundary_token = env_str("KORITH_AMF_PREFIX_BOUNDARY_TOKEN", e.amf_prefix_boundary_token)
        e.amf_tenant_isolation = env_bool("KORITH_AMF_TENANT_ISOLATION", False)
        e.amf_normalize_whitespace = env_bool("KORITH_AMF_NORMALIZE_WHITESPACE", False)
        e.amf_normalize_unicode = env_bool("KORITH_AMF_NORMALIZE_UNICODE", False)
        e.amf_prompt_collapse_blanks = env_bool("KORITH_AMF_PROMPT_COLLAPSE_BLANKS", False)
        e.amf_prompt_strip_outer = env_bool("KORITH_AMF_PROMPT_STRIP_OUTER", False)
        e.amf_canonicalize_template_json = env_bool("KORITH_AMF_CANONICALIZE_TEMPLATE_JSON", False)
        e.amf_vram_first = env_bool("KORITH_AMF_VRAM_FIRST", True)
        e.amf_sync_save = env_bool("KORITH_AMF_SYNC_SAVE", False)
        e.vram_cache_device = env_str("KORITH_VRAM_CACHE_DEVICE", e.vram_cache_device)
        e.vram_cache_gb = env_float("KORITH_VRAM_CACHE_GB", 0.0, lo=0.0)
        e.vram_pool_gb = env_float("KORITH_VRAM_POOL_GB", 0.0, lo=0.0)
        q = env_str("KORITH_VRAM_POOL_QUANT", e.vram_pool_quant).lower()
        if q in ("fp8", "int4", "raw", "bf16"):
            e.vram_pool_quant = q
        e.lmcache_fallback = env_bool("AXROPUS_LMCACHE_FALLBACK", False)
        e.promote_lmcache_hits = env_bool("AXROPUS_PROMOTE_LMCACHE_HITS", True)
        e.lmcache_write_through = env_bool("AXROPUS_LMCACHE_WRITE_THROUGH", False)
        e.lmcache_lookup_timeout_ms = env_int("AXROPUS_LMCACHE_LOOKUP_TIMEOUT_MS", e.lmcache_lookup_timeout_ms, minimum=0)
        e.kv_fp8 = env_bool("KORITH_KV_FP8", False)
        e.kv_type_k = env_str("KORITH_KV_TYPE_K", "")
        e.kv_type_v = env_str("KORITH_KV_TYPE_V", "")
        e.tensor_split = env_str("KORITH_TENSOR_SPLIT", "")
        e.main_gpu = env_int("KORITH_MAIN_GPU", 0, minimum=0)
        e.n_ctx = env_int("KORITH_N_CTX", e.n_ctx, minimum=1)
        e.n_batch = env_int("KORITH_N_BATCH", e.n_batch, minimum=1)
        e.n_seq_max = env_int("KORITH_N_SEQ_MAX", e.n_seq_max, minimum=1)
        e.allow_n_ctx_fallback = env_bool("KORITH_ALLOW_N_CTX_FALLBACK", True)
        e.cuda_graphs = env_bool("KORITH_CUDA_GRAPHS", True)
        e.cuda_graph_cache_size = min(64, max(1, env_int("KORITH_CUDA_GRAPH_CACHE_SIZE", 4)))
        e.cuda_graph_capture = env_bool("KORITH_CUDA_GRAPH_CAPTURE", False)
        e.batch_tokens = env_int("KORITH_BATCH_TOKENS", e.batch_tokens, minimum=1)
        e.draft_model = os.environ.get("KORITH_DRAFT_MODEL_PATH") or os.environ.get("KORITH_DRAFT_MODEL", "")
        e.spec_v2 = env_bool("KORITH_SPEC_V2", False)
        e.spec_v3 = env_bool("KORITH_SPEC_V3", False)
        e.spec_depth = env_int("KORITH_SPEC_DEPTH", 0, minimum=0)
        e.spec_k = env_int("KORITH_SPEC_K", e.spec_k, minimum=1)
        e.spec_min_accept = env_float("KORITH_SPEC_MIN_ACCEPT", 0.0, 0.0, 1.0)
        e.spec_allow_exec = env_bool("KORITH_SPEC_ALLOW_EXEC", True)
        e.spec_allow_commit = env_bool("KORITH_SPEC_ALLOW_COMMIT", True)
        e.spec_pause = env_bool("KORITH_SPEC_PAUSE", False)
        e.max_depth = env_int("KORITH_MAX_DEPTH", e.max_depth, minimum=1)
        e.scheduler_lib = env_str("KORITH_SCHEDULER_LIB", "")
        e.sched_decode_first = env_bool("KORITH_VLLM_DECODE_FIRST", True)
        e.sched_adaptive_budget = env_bool("KORITH_VLLM_ADAPTIVE_BUDGET", True)
        e.sched_budget_scale_decode = env_float("KORITH_VLLM_BUDGET_SCALE_DECODE", 1.0, lo=0.0)
        e.sched_decode_ratio_threshold = env_float("KORITH_VLLM_DECODE_RATIO_THRESHOLD", 0.5, 0.0, 1.0)
        e.sched_min_scheduled_tokens = env_int("KORITH_VLLM_MIN_SCHEDULED_TOKENS", 1, minimum=1)
        e.sched_starvation_s = env_float("KORITH_VLLM_STARVATION_S", 2.0, lo=0.0)
        e.sched_prefill_penalty = env_float("KORITH_VLLM_PREFILL_PENALTY", 0.0)
        e.sched_short_decode_bonus = env_float("KORITH_VLLM_SHORT_DECODE_BONUS", 0.0)
        e.sched_decode_full_budget_on_hit = env_bool("KORITH_VLLM_DECODE_FULL_BUDGET_ON_HIT", True)
        e.sched_trace_path = env_str("KORITH_VLLM_SCHED_TRACE_PATH", "")
        e.sched_trace_every = env_int("KORITH_VLLM_SCHED_TRACE_EVERY", 0, minimum=0)
        e.engine_events_path = env_str("KORITH_ENGINE_EVENTS_PATH", "")
        e.engine_metrics_path = env_str("KORITH_ENGINE_METRICS_PATH", "")
        e.mf_snapshot_in = env_str("KORITH_MF_SNAPSHOT_IN", "")
        e.mf_snapshot_out = env_str("KORITH_MF_SNAPSHOT_OUT", "")
        return c

    @property
    def kv_cache_dtype(self) -> str:
        """Live paged-KV storage format: ``KORITH_KV_FP8`` -> fp8, ``KORITH_KV_TYPE_K``
        of q4/int4 -> int4, default bf16."""
        k = (self.kv_type_k or "").lower()
        if k in ("int4", "q4", "q4_0", "q4_1"):
            return "int4"
        if self.kv_fp8 or k in ("fp8", "q8_0", "f8"):
            return "fp8"
        return "bf16"

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


__all__ = ["AxropusConfig", "KorithConfig", "env_bool", "env_int", "env_float", "env_str"]
