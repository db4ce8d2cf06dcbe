"""Runtime helpers of the control plane: the speculative-depth controller, the decode
output cache, replay / speculation governance and the platform config loader.

* :class:`SpecKController` -- draft depth k per worker: an exponential moving average
  (alpha 0.2) of the per-step acceptance rate raises k above 0.85 and lowers it below
  0.65, within [2, 12] (default 4); it also books the decode time speculation saved
  (accepted tokens beyond the first, priced at the measured non-speculative rate) and
  its overhead. Jobs whose policy forbids speculation, or whose backend can neither
  verify tokens nor expose logits, run without it.
* :class:`DecodeCache` -- SQLite cache of finished outputs keyed by
  (org, backend, fingerprint, prompt hash, sampling hash): a deterministic job that was
  already answered is served without running the model.
* :class:`ReplayGovernor` -- per-fingerprint replay switch in the ledger: restores
  that keep costing more than they save (``KORITH_NEGATIVE_ROI_MAX`` in a row) or a
  snapshot that fails validation disable replay for ``KORITH_NEGATIVE_ROI_COOLDOWN_MS``;
  :class:`SpecGovernor` does the same for speculation after
  ``KORITH_SPEC_DISABLE_AFTER_N`` steps below ``KORITH_SPEC_MIN_ACCEPT``.
* :func:`load_platform_config` / :func:`apply_config_to_env` -- a YAML/JSON platform
  file mapped onto the ``KORITH_*`` variables (set variables win).

Reference: platform/runtime/spec_decode.py:6-134, platform/runtime/decode_cache_store.py,
platform/runtime/config.py:34-225 (file keys and variable names), cluster_worker.py
replay/spec governance.
"""
from __future__ import annotations

import json
import os
import sqlite3
import threading
import time
from pathlib import Path
from typing import Any, Dict, Optional

from .observability import utc_now


class SpecKController:
    MIN_K, MAX_K, DEFAULT_K = 2, 12, 4
    RAISE_ABOVE, LOWER_BELOW, ALPHA = 0.85, 0.65, 0.2

    def __init__(self, k: Optional[int] = None):
        self.k = int(k or self.DEFAULT_K)
        self.enabled = False
        self.proposed = self.accepted = 0
        self.ema: Optional[float] = None
        self.saved_ms = self.overhead_ms = 0.0

    def gate(self, capabilities: Dict[str, bool], policy: Dict[str, Any]) -> Dict[str, Any]:
        if not policy.get("allow_spec", False):
            return {"enabled": False, "reason": "policy_disabled", "k": 0}
        if not (capabilities.get("VERIFY_TOKENS") or capabilities.get("LOGITS_ACCESS")):
            return {"enabled": False, "reason": "capability_missing", "k": 0}
        self.enabled = True
        return {"enabled": True, "reason": "ok", "k": self.k}

    def update(self, proposed: int, accepted: int, spec_ms: float = 0.0, baseline_tok_s: float = 0.0) -> None:
        self.proposed += proposed
        self.accepted += accepted
        if proposed > 0:
            rate = accepted / proposed
            self.ema = rate if self.ema is None else self.ema + self.ALPHA * (rate - self.ema)
            if self.ema > self.RAISE_ABOVE:
                self.k = min(self.MAX_K, self.k + 1)
            elif self.ema < self.LOWER_BELOW:
                self.k = max(self.MIN_K, self.k - 1)
        self.overhead_ms += max(0.0, spec_ms)
        if accepted > 1 and baseline_tok_s > 0:
            self.saved_ms += max(0.0, (accepted - 1) * 1e3 / baseline_tok_s - spec_ms)

    def metrics(self) -> Dict[str, Any]:
        return {"enabled": self.enabled, "k": self.k,
                "acceptance_rate": round(self.accepted / self.proposed, 4) if self.proposed else 0.0,
                "accept_ema": round(self.ema or 0.0, 4), "tokens_proposed": self.proposed,
                "tokens_accepted": self.accepted, "decode_ms_saved": round(self.saved_ms, 2),
                "spec_overhead_ms": round(self.overhead_ms, 2)}


class DecodeCache:
    def __init__(self, path: str = ":memory:"):
        if path != ":memory:":
            Path(path).parent.mkdir(parents=True, exist_ok=True)
        self._mu = threading.Lock()
        self._c = sqlite3.connect(path, check_same_thread=False, timeout=10.0)
        self._c.execute("CREATE TABLE IF NOT EXISTS decode_cache (org_id TEXT NOT NULL, backend_id TEXT NOT NULL, "
                        "fingerprint_hash TEXT NOT NULL, prompt_hash TEXT NOT NULL, sampling_hash TEXT NOT NULL, "
                        "output_text TEXT NOT NULL, tokens_out INTEGER NOT NULL, decode_ms REAL NOT NULL DEFAULT 0, "
                        "total_ms REAL NOT NULL DEFAULT 0, updated_at REAL NOT NULL, PRIMARY KEY (org_id, "
                        "backend_id, fingerprint_hash, prompt_hash, sampling_hash))")
        self._c.commit()

    def get(self, *, org_id: str, backend_id: str, fingerprint_hash: str, prompt_hash: str,
            sampling_hash: str) -> Optional[Dict[str, Any]]:
        with self._mu:
            r = self._c.execute("SELECT output_text, tokens_out, decode_ms, total_ms, updated_at FROM decode_cache "
                                "WHERE org_id=? AND backend_id=? AND fingerprint_hash=? AND prompt_hash=? AND "
                                "sampling_hash=?", (org_id, backend_id, fingerprint_hash, prompt_hash,
                                                    sampling_hash)).fetchone()
        if r is None:
            return None
        return {"output_text": r[0], "tokens_out": int(r[1]), "decode_ms": float(r[2]), "total_ms": float(r[3]),
                "updated_at": float(r[4])}

    def put(self, *, org_id: str, backend_id: str, fingerprint_hash: str, prompt_hash: str, sampling_hash: str,
            output_text: str, tokens_out: int, decode_ms: float = 0.0, total_ms: float = 0.0) -> None:
        with self._mu:
            self._c.execute("INSERT OR REPLACE INTO decode_cache VALUES (?,?,?,?,?,?,?,?,?,?)",
                            (org_id, backend_id, fingerprint_hash, prompt_hash, sampling_hash, output_text,
                             int(tokens_out), float(decode_ms), float(total_ms), time.time()))
            self._c.commit()


def _envf(name: str, default: float) -> float:
    try:
        return float(os.environ.get(name, "") or default)
    except ValueError:
        return default


class ReplayGovernor:
    def __init__(self, ledger, negative_roi_max: Optional[int] = None, cooldown_ms: Optional[float] = None):
        self.ledger = ledger
        self.max_streak = int(negative_roi_max or _envf("KORITH_NEGATIVE_ROI_MAX", 3))
        self.cooldown_s = (cooldown_ms if cooldown_ms is not None else _envf("KORITH_NEGATIVE_ROI_COOLDOWN_MS",
                                                                             600_000)) / 1e3

    def status(self, fp: str, now: Optional[float] = None) -> Dict[str, Any]:
        g = self.ledger.get_replay_governance(fp) or {}
        t = time.time() if now is None else now
        disabled = bool(g.get("replay_disabled")) and t < float(g.get("cooldown_until", 0.0))
        return {"fingerprint_hash": fp, "replay_allowed": not disabled, "replay_disabled": disabled,
                "disabled_reason": g.get("disabled_reason") if disabled else None,
                "negative_roi_streak": int(g.get("negative_roi_streak", 0) or 0),
                "corruption_detected": bool(g.get("corruption_detected", 0)),
                "cooldown_until": float(g.get("cooldown_until", 0.0) or 0.0)}

    def record(self, fp: str, saved_ms: float, corrupted: bool = False, now: Optional[float] = None) -> Dict[str, Any]:
        t = time.time() if now is None else now
        g = self.ledger.get_replay_governance(fp) or {}
        streak = 0 if saved_ms > 0 and not corrupted else int(g.get("negative_roi_streak", 0) or 0) + 1
        disable = corrupted or streak >= self.max_streak
        reason = "snapshot_corrupted" if corrupted else ("negative_roi" if disable else None)
        self.ledger.upsert_replay_governance(fp, int(disable), reason, utc_now() if disable else None,
                                             t + self.cooldown_s if disable else 0.0, 0 if disable else streak,
                                             int(corrupted or g.get("corruption_detected", 0)), 0, utc_now())
        return self.status(fp, t)


class SpecGovernor:
    def __init__(self, ledger, min_accept: Optional[float] = None, disable_after_n: Optional[int] = None,
                 cooldown_s: float = 600.0):
        self.ledger = ledger
        self.min_accept = min_accept if min_accept is not None else _envf("KORITH_SPEC_MIN_ACCEPT", 0.3)
        self.after_n = int(disable_after_n or _envf("KORITH_SPEC_DISABLE_AFTER_N", 3))
        self.cooldown_s = cooldown_s

    def allowed(self, fp: str, now: Optional[float] = None) -> bool:
        g = self.ledger.get_spec_governance(fp) or {}
        t = time.time() if now is None else now
        return not (g.get("spec_disabled") and t < float(g.get("cooldown_until", 0.0)))

    def record(self, fp: str, org_id: str, acceptance: float, now: Optional[float] = None) -> bool:
        t = time.time() if now is None else now
        g = self.ledger.get_spec_governance(fp) or {}
        streak = int(g.get("bad_accept_streak", 0) or 0) + 1 if acceptance < self.min_accept else 0
        disable = streak >= self.after_n
        self.ledger.upsert_spec_governance(fp, org_id, int(disable), "low_acceptance" if disable else None,
                                           t + self.cooldown_s if disable else 0.0, 0 if disable else streak,
                                           utc_now())
        return not disable


# ---------------------------------------------------------------------- config file -> environment
CONFIG_ENV = {
    "ledger.backend": "KORITH_LEDGER_BACKEND",
    "ledger.sqlite_path": "KORITH_PLATFORM_DB",
    "ledger.postgres_dsn": "KORITH_LEDGER_DSN",
    "artifacts.backend": "KORITH_ARTIFACT_BACKEND",
    "artifacts.local_path": "KORITH_PLATFORM_ARTIFACTS",
    "artifacts.s3_bucket": "KORITH_S3_BUCKET",
    "artifacts.s3_prefix": "KORITH_S3_PREFIX",
    "artifacts.s3_endpoint": "KORITH_S3_ENDPOINT",
    "artifacts.minio_endpoint": "KORITH_MINIO_ENDPOINT",
    "artifacts.minio_access_key": "KORITH_MINIO_ACCESS_KEY",
    "artifacts.minio_secret_key": "KORITH_MINIO_SECRET_KEY",
    "artifacts.minio_bucket": "KORITH_MINIO_BUCKET",
    "artifacts.minio_prefix": "KORITH_MINIO_PREFIX",
    "artifacts.minio_secure": "KORITH_MINIO_SECURE",
    "queue.backend": "KORITH_QUEUE_BACKEND",
    "queue.sqlite_path": "KORITH_QUEUE_DB",
    "queue.redis_url": "KORITH_REDIS_URL",
    "queue.stream_prefix": "KORITH_STREAM_PREFIX",
    "queue.consumer_group": "KORITH_STREAM_CONSUMER_GROUP",
    "queue.nats_url": "KORITH_NATS_URL",
    "queue.sqs_url": "KORITH_SQS_URL",
    "queue.inflight_stale_s": "KORITH_QUEUE_INFLIGHT_STALE_S",
    "cluster.node_id": "KORITH_NODE_ID",
    "cluster.node_host": "KORITH_NODE_HOST",
    "cluster.node_router_port": "KORITH_NODE_ROUTER_PORT",
    "cluster.registry.sqlite_path": "KORITH_NODE_REGISTRY_DB",
    "cluster.registry.redis_url": "KORITH_NODE_REGISTRY_REDIS_URL",
    "cluster.snapshot_index.redis_url": "KORITH_SNAPSHOT_INDEX_REDIS_URL",
    "cluster.snapshot_bw_mbps": "KORITH_SNAPSHOT_BW_MBPS",
    "cluster.snapshot_rtt_ms": "KORITH_SNAPSHOT_RTT_MS",
    "cluster.transfer_vs_recompute_threshold": "KORITH_TRANSFER_VS_RECOMPUTE_THRESHOLD",
    "registry.sqlite_path": "KORITH_REGISTRY_DB",
    "runtime.backend_id": "KORITH_DEFAULT_BACKEND_ID",
    "runtime.model_id": "KORITH_DEFAULT_MODEL_ID",
    "runtime.model_path": "KORITH_DEFAULT_MODEL_PATH",
    "runtime.model_endpoint": "KORITH_DEFAULT_MODEL_ENDPOINT",
    "runtime.scheduler.hit_priority": "KORITH_HIT_PRIORITY",
    "runtime.scheduler.miss_priority": "KORITH_MISS_PRIORITY",
    "runtime.scheduler.spec_priority": "KORITH_SPEC_PRIORITY",
    "runtime.scheduler.negative_roi_max": "KORITH_NEGATIVE_ROI_MAX",
    "runtime.scheduler.negative_roi_cooldown_ms": "KORITH_NEGATIVE_ROI_COOLDOWN_MS",
    "runtime.engine.accel_enabled": "KORITH_ACCEL_ENABLED",
    "runtime.engine.cuda_device": "KORITH_CUDA_DEVICE",
    "runtime.engine.kv_layout_version": "KORITH_KV_LAYOUT_VERSION",
    "runtime.spec.enabled": "KORITH_SPEC_ENABLED",
    "runtime.spec.k": "KORITH_SPEC_K",
    "runtime.spec.min_accept": "KORITH_SPEC_MIN_ACCEPT",
    "runtime.spec.disable_after_n": "KORITH_SPEC_DISABLE_AFTER_N",
    "gateway.rate_limit.backend": "KORITH_RATE_LIMIT_BACKEND",
    "gateway.rate_limit.sqlite_path": "KORITH_RATE_LIMIT_DB",
    "gateway.rate_limit.redis_url": "KORITH_REDIS_URL",
    "gateway.rate_limit.burst_factor": "KORITH_RATE_LIMIT_BURST",
    "security.api_key_salt": "KORITH_API_KEY_SALT",
}


def load_platform_config(path: Optional[str]) -> Dict[str, Any]:
    if not path or not Path(path).exists():
        return {}
    raw = Path(path).read_text(encoding="utf-8")
    if Path(path).suffix.lower() == ".json":
        data = json.loads(raw)
    else:
        import yaml

        data = yaml.safe_load(raw)
    return data if isinstance(data, dict) else {}


def _deep_get(d: Dict[str, Any], dotted: str) -> Any:
    cur: Any = d
    for part in dotted.split("."):
        if not isinstance(cur, dict) or part not in cur:
            return None
        cur = cur[part]
    return cur


def apply_config_to_env(config: Dict[str, Any], environ=None) -> Dict[str, str]:
    """Copy the file's values onto unset ``KORITH_*`` variables; returns what was set.
    Unknown top-level sections are an error (a typo would otherwise be ignored)."""
    env = os.environ if environ is None else environ
    known = {k.split(".")[0] for k in CONFIG_ENV}
    bad = [k for k in config if k not in known]
    if bad:
        raise ValueError(f"unknown config sections: {sorted(bad)}")
    out = {}
    for dotted, name in CONFIG_ENV.items():
        v = _deep_get(config, dotted)
        if v is None or env.get(name):
            continue
        env[name] = out[name] = str(v).lower() if isinstance(v, bool) else str(v)
    return out
