"""Decisions of the policy layer and how they reach the serving path.

* :class:`Decision` -- one decision for prefill / cache admission and for decode
  (speculative depth, draft temperature, back-pressure, pre-warm list, fleet hints), with
  the reference's field names so a model prompted with them answers in this shape.
* :class:`AdaptivePolicy` -- the default decider, sub-millisecond and local: per-tenant
  EMAs of hit rate and ROI (the ROI EMA seeded by the first evidence, admission kept on until
  there is some); cache admission with a hysteresis band (on below
  ``ADMIT - BAND`` turns off, off above ``ADMIT + BAND`` turns on, so it does not flap);
  speculative depth by UCB1 over the arms ``DEPTHS`` (entropy picks the depth until every
  arm has data); rewards scaled by a streak multiplier (doubles on each correct admission,
  halves on a wrong one, capped); pre-warm list from per-tenant prefix hit counts. An
  optional model (:class:`EndpointModel` or anything with ``decide(vector)``) is asked only
  when the tenant's hit rate sits in an uncertainty band, or first when ``model_primary``.
* :class:`EndpointModel` -- asks an OpenAI-compatible chat endpoint (this framework's own
  server, or any other) for a decision as JSON, validates it, and falls back to the rules on
  any error or timeout.
* :class:`DecisionExecutor` -- applies a decision with safety clamps and fails closed: an
  invalid or out-of-policy decision changes nothing. It sets the worker's speculative depth
  controller, the AMF manager's capture switch, and a back-pressure fraction the admission
  path reads; with ``config_path`` it also writes the decode settings as JSON for engines in
  other processes.

Reference: platform/reasoning/reasoning_model.py:216-326 (decision fields),
adaptive_engine.py:60-416 (constants and algorithm), nemoclaw_model.py:88 (endpoint model),
decision_executor.py:102-300 (clamped application, decode config file).
"""
from __future__ import annotations

import json
import math
import os
import threading
import time
import urllib.request
from collections import defaultdict
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import numpy as np

from .state import Slot

DEPTHS = (2, 4, 6, 8, 12, 16)
UCB_C = 1.4
ADMIT, BAND = 0.30, 0.08
EMA_ALPHA = 0.15
PREWARM_MIN_HITS = 3
MULT_MAX, MULT_DECAY = 64.0, 0.5
UNCERTAIN = (0.35, 0.65)


@dataclass
class Decision:
    cache_admission: bool = True
    admission_priority: float = 0.5
    eviction_target: Optional[str] = None
    pre_warm_predictions: List[str] = field(default_factory=list)
    route_decision: Optional[str] = None
    batch_group: Optional[str] = None
    throttle_back_pressure: float = 0.0
    inference_ms: float = 0.0
    is_fallback: bool = False
    domain: str = "unified"
    prefer_local_restore: bool = True
    cross_node_restore_target: Optional[str] = None
    persist_priority: float = 0.0
    replicate_to_nodes: List[str] = field(default_factory=list)
    evict_hint_nodes: List[str] = field(default_factory=list)
    spec_decode_enable: bool = True
    spec_decode_depth: int = 4
    spec_mode: str = "v2_clean"
    spec_v3_block_size: int = 8
    draft_temperature: float = 0.8
    kv_compression_enable: bool = False
    kv_compression_ratio: float = 1.0
    decode_batch_priority: int = 2
    early_stop_confidence: float = 0.0
    cuda_graph_hint: bool = True
    adaptive_depth_override: bool = False

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "Decision":
        """Accepts the flat form or the reference's nested ``{"prefill": …, "decode": …, "dynamo": …}``."""
        flat: Dict[str, Any] = {}
        for k, v in d.items():
            if isinstance(v, dict) and k in ("prefill", "decode", "dynamo"):
                flat.update(v)
            else:
                flat[k] = v
        names = set(cls.__dataclass_fields__)
        return cls(**{k: v for k, v in flat.items() if k in names})

    def validate(self) -> List[str]:
        """Reasons this decision is out of policy (empty: valid)."""
        bad = []
        for name, lo, hi in (("admission_priority", 0, 1), ("throttle_back_pressure", 0, 1),
                             ("persist_priority", 0, 1), ("draft_temperature", 0, 2),
                             ("kv_compression_ratio", 0.1, 1), ("early_stop_confidence", 0, 1)):
            x = getattr(self, name)
            if not isinstance(x, (int, float)) or not math.isfinite(x) or not lo <= x <= hi:
                bad.append(f"{name}={x!r} outside [{lo}, {hi}]")
        if not isinstance(self.spec_decode_depth, int) or not 1 <= self.spec_decode_depth <= 16:
            bad.append(f"spec_decode_depth={self.spec_decode_depth!r} outside [1, 16]")
        if self.spec_mode not in ("v2_clean", "v3_block", "disabled"):
            bad.append(f"spec_mode={self.spec_mode!r}")
        if not 4 <= int(self.spec_v3_block_size) <= 32:
            bad.append(f"spec_v3_block_size={self.spec_v3_block_size!r} outside [4, 32]")
        if not 1 <= int(self.decode_batch_priority) <= 4:
            bad.append(f"decode_batch_priority={self.decode_batch_priority!r} outside [1, 4]")
        return bad


def _ema(cur: float, new: float, a: float = EMA_ALPHA) -> float:
    return cur * (1 - a) + new * a


@dataclass
class _Arm:
    pulls: int = 0
    reward: float = 0.0

    def ucb(self, total: int) -> float:
        if self.pulls == 0:
            return float("inf")
        return self.reward / self.pulls + UCB_C * math.sqrt(math.log(total + 1) / self.pulls)


@dataclass
class _Tenant:
    hit_ema: float = 0.0
    roi_ema: float = 0.0
    admit: bool = True
    arms: Dict[int, _Arm] = field(default_factory=lambda: {d: _Arm() for d in DEPTHS})
    pulls: int = 0
    hits: Dict[str, int] = field(default_factory=dict)
    streak: int = 0
    mult: float = 1.0
    requests: int = 0
    roi_seen: bool = False


class AdaptivePolicy:
    def __init__(self, model=None, uncertain: Tuple[float, float] = UNCERTAIN, model_primary: bool = False,
                 max_prefix_memory: int = 10000):
        self.model, self.uncertain, self.model_primary = model, uncertain, model_primary
        self.max_prefix_memory = max_prefix_memory
        self._t: Dict[str, _Tenant] = defaultdict(_Tenant)
        self._mu = threading.Lock()
        self.stat = {"decisions": 0, "local": 0, "model": 0, "model_failures": 0, "reward": 0.0}

    def decide(self, v: np.ndarray, tenant_id: str = "default", prefix_hash: str = "") -> Decision:
        t0 = time.perf_counter()
        with self._mu:
            self.stat["decisions"] += 1
            t = self._t[tenant_id]
            t.requests += 1
            t.hit_ema = _ema(t.hit_ema, float(v[Slot.HIT_RATE]))
            live_roi = float(v[Slot.ROI_EMA_NORM]) * 10.0
            if t.roi_seen:
                t.roi_ema = _ema(t.roi_ema, live_roi)
            elif live_roi != 0.0:  # the first ROI evidence seeds the EMA instead of averaging with 0
                t.roi_seen, t.roi_ema = True, live_roi
            ask = self.model is not None and (self.model_primary or self.uncertain[0] <= t.hit_ema <= self.uncertain[1])
        if ask:
            try:
                d = self.model.decide(v)
                if not d.is_fallback and not d.validate():
                    with self._mu:
                        self.stat["model"] += 1
                    return d
            except Exception:
                pass
            with self._mu:
                self.stat["model_failures"] += 1
        with self._mu:
            self.stat["local"] += 1
            # hysteresis admission on the ROI EMA; a tenant with no ROI evidence yet stays admitted
            if t.roi_seen:
                if t.admit and t.roi_ema < ADMIT - BAND:
                    t.admit = False
                elif not t.admit and t.roi_ema > ADMIT + BAND:
                    t.admit = True
            ent = float(v[Slot.ENTROPY_EMA])
            if t.pulls < 2 * len(DEPTHS):
                depth = 8 if ent < 0.3 else 6 if ent < 0.6 else 4
            else:
                depth = max(DEPTHS, key=lambda d: t.arms[d].ucb(t.pulls))
            thr = 0.0
            if v[Slot.MISS_STREAK_NORM] > 0.3:
                thr += min(float(v[Slot.MISS_STREAK_NORM]) * 0.3, 0.3)
            if v[Slot.STORAGE_UTIL] > 0.85:
                thr += (float(v[Slot.STORAGE_UTIL]) - 0.85) * 2.0
            if v[Slot.MEMORY_PRESSURE] > 0.80:
                thr += (float(v[Slot.MEMORY_PRESSURE]) - 0.80) * 1.5
            warm = sorted(((h, n) for h, n in t.hits.items() if h != prefix_hash and n >= PREWARM_MIN_HITS),
                          key=lambda x: -x[1])[:3]
            return Decision(cache_admission=t.admit, admission_priority=max(0.0, min(1.0, t.hit_ema)),
                            pre_warm_predictions=[h for h, _ in warm], throttle_back_pressure=round(min(thr, 0.5), 3),
                            spec_decode_depth=depth, draft_temperature=round(0.5 + ent * 0.6, 2),
                            inference_ms=(time.perf_counter() - t0) * 1e3)

    def record_outcome(self, prefix_hash: str = "", tenant_id: str = "default", spec_depth: int = 4,
                       admitted: bool = True, was_hit: bool = False, acceptance_rate: float = 0.0) -> float:
        """Feed back what happened; returns the scaled reward given to the depth arm."""
        with self._mu:
            t = self._t[tenant_id]
            if was_hit and admitted:
                t.streak += 1
                t.mult = min(MULT_MAX, 2.0 ** t.streak)
            else:
                t.streak = 0
                t.mult = max(1.0, t.mult * MULT_DECAY)
            if prefix_hash and was_hit:
                t.hits[prefix_hash] = t.hits.get(prefix_hash, 0) + 1
                if len(t.hits) > self.max_prefix_memory:
                    del t.hits[next(iter(t.hits))]
            r = 0.0
            if spec_depth in t.arms:
                r = (acceptance_rate if was_hit else -0.2) * t.mult
                t.arms[spec_depth].pulls += 1
                t.arms[spec_depth].reward += r
                t.pulls += 1
                self.stat["reward"] += r
            return r

    def tenant_stats(self, tenant_id: str = "default") -> Dict[str, Any]:
        with self._mu:
            t = self._t[tenant_id]
            return {"hit_ema": t.hit_ema, "roi_ema": t.roi_ema, "admit": t.admit, "streak": t.streak,
                    "multiplier": t.mult, "arm_pulls": {d: a.pulls for d, a in t.arms.items()}}


class EndpointModel:
    """Decision from an OpenAI-compatible chat endpoint; any failure returns a fallback."""

    SYSTEM = ("You control a KV-cache-aware LLM serving node. Given the state vector (slot name -> value), "
              "answer with ONE JSON object with the fields of the decision: " + ", ".join(Decision.__dataclass_fields__)
              + ". No prose.")

    def __init__(self, base_url: str, model: str = "default", api_key: str = "", timeout_s: float = 2.0):
        self.url = base_url.rstrip("/") + "/v1/chat/completions"
        self.model, self.api_key, self.timeout_s = model, api_key, timeout_s

    @staticmethod
    def _named(v: np.ndarray) -> Dict[str, float]:
        return {k: round(float(v[i]), 4) for k, i in vars(Slot).items() if k.isupper() and i < len(v)}

    def decide(self, v: np.ndarray) -> Decision:
        t0 = time.perf_counter()
        body = {"model": self.model, "temperature": 0.0, "max_tokens": 512,
                "messages": [{"role": "system", "content": self.SYSTEM},
                             {"role": "user", "content": json.dumps(self._named(v))}]}
        req = urllib.request.Request(self.url, json.dumps(body).encode(), {"Content-Type": "application/json",
                                                                          **({"Authorization": f"Bearer {self.api_key}"}
                                                                             if self.api_key else {})})
        try:
            with urllib.request.urlopen(req, timeout=self.timeout_s) as r:
                text = json.loads(r.read())["choices"][0]["message"]["content"]
            s, e = text.index("{"), text.rindex("}") + 1
            d = Decision.from_dict(json.loads(text[s:e]))
            d.inference_ms = (time.perf_counter() - t0) * 1e3
            if d.validate():
                raise ValueError("; ".join(d.validate()))
            return d
        except Exception:
            return Decision(is_fallback=True, inference_ms=(time.perf_counter() - t0) * 1e3)


class DecisionExecutor:
    """Applies decisions to this node. Clamps: depth to the controller's [MIN_K, MAX_K] and to
    at most 3 while the acceptance EMA is below ``low_acceptance``; back-pressure to
    [0, ``max_throttle``]. An invalid decision is rejected whole (counted, nothing changed)."""

    def __init__(self, spec_controller=None, amf=None, config_path: Optional[str] = None, max_throttle: float = 0.5,
                 low_acceptance: float = 0.3):
        self.spec, self.amf, self.config_path = spec_controller, amf, config_path
        self.max_throttle, self.low_acceptance = max_throttle, low_acceptance
        self.back_pressure = 0.0
        self.applied: Optional[Decision] = None
        self.stat = {"applied": 0, "rejected": 0, "clamped": 0}

    def execute(self, d: Decision, v: Optional[np.ndarray] = None) -> Dict[str, Any]:
        bad = d.validate()
        if bad:
            self.stat["rejected"] += 1
            return {"applied": False, "reasons": bad}
        depth = d.spec_decode_depth
        if v is not None and float(v[Slot.ACCEPTANCE_EMA]) < self.low_acceptance and float(v[Slot.CURRENT_SPEC_DEPTH]) > 0:
            depth = min(depth, 3)
        if self.spec is not None:
            depth = max(self.spec.MIN_K, min(self.spec.MAX_K, depth))
            self.spec.k = depth
        clamped = depth != d.spec_decode_depth
        self.stat["clamped"] += int(clamped)
        self.back_pressure = max(0.0, min(self.max_throttle, d.throttle_back_pressure))
        if self.amf is not None and hasattr(self.amf, "capture_enabled"):
            self.amf.capture_enabled = bool(d.cache_admission)
        if self.config_path:
            cfg = {"spec_decode_enable": d.spec_decode_enable and d.spec_mode != "disabled", "spec_depth": depth,
                   "spec_mode": d.spec_mode, "spec_v3_block_size": int(d.spec_v3_block_size),
                   "draft_temperature": d.draft_temperature, "decode_batch_priority": int(d.decode_batch_priority),
                   "cuda_graph_hint": d.cuda_graph_hint, "written_at": time.time()}
            tmp = self.config_path + ".tmp"
            with open(tmp, "w") as f:
                json.dump(cfg, f)
            os.replace(tmp, self.config_path)  # readers never see a partial file
        self.applied = d
        self.stat["applied"] += 1
        return {"applied": True, "spec_depth": depth, "clamped": clamped, "back_pressure": self.back_pressure}


def read_decode_config(path: str) -> Dict[str, Any]:
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}
