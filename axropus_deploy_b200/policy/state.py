"""The policy layer's view of a serving node: a fixed-width float32 state vector sampled
from the engine, the AMF tiers, the worker queues and the GPU's power draw.

Slot numbers are a contract between the collector and every decision maker (rules,
bandit, learned policy, an external model that reads the vector as JSON), so they keep the
reference's assignment: 0-31 prefix cache / fleet, 32-53 decode and speculative decoding,
54-69 disaggregated-serving fleet signals; width 72. Values are normalised to about
[0, 1]; rates are per second over a sliding window.

:class:`PowerSampler` reads board power through NVML (read-only: it queries
``nvmlDeviceGetPowerUsage`` and the enforced limit, and changes nothing on the GPU); tests
hand it a fake NVML module.

Reference: platform/reasoning/metrics_collector.py:80-156 (slot table), :202-292 (polling
collector) and python/power.py:40-140 (NVML power sampling).
"""
from __future__ import annotations

import math
import threading
import time
from collections import deque
from typing import Any, Callable, Dict, Optional

import numpy as np

WIDTH = 72


class Slot:
    HIT_DELTA, MISS_DELTA, HIT_RATE, TOKENS_SAVED_DELTA, SAVINGS_MS_DELTA, RESTORE_MS_AVG = range(6)
    EVICTION_RATE, ADMISSION_RATE, REJECTION_RATE, FAILURE_RATE, STORAGE_UTIL, EVICTION_PRESSURE = range(6, 12)
    ENTRY_COUNT_NORM, HOT_ENTRY_RATIO, COLD_ENTRY_RATIO, INSTANT_TPS_NORM, ROLLING_TPS_NORM = range(12, 17)
    NODE_COUNT, AVG_NODE_HIT_RATE, AVG_NODE_WARMTH, TOTAL_CACHE_ENTRIES, TOTAL_CACHE_GB = range(17, 22)
    REQUEST_RATE, HIT_STREAK_NORM, MISS_STREAK_NORM, REUSE_RATIO, UNIQUE_PREFIXES_NORM = range(22, 27)
    HIT_QUEUE_NORM, MISS_QUEUE_NORM, ROI_EMA_NORM, MEMORY_PRESSURE, DECODE_LATENCY_NORM = range(27, 32)
    ACCEPTANCE_EMA, ACCEPTANCE_VARIANCE, CURRENT_SPEC_DEPTH, ENTROPY_EMA, TPS_CURRENT, TPS_DELTA = range(32, 38)
    TOKENS_COMMITTED_NODECODE, TOKENS_DECODED_NORMALLY, SPEC_PROFIT_RATIO, SPEC_BAD_STREAK = range(38, 42)
    SPEC_COOLDOWN_REMAINING, LANE_CURRENT, LANE_HOLD_REMAINING, STARVATION_COUNTER = range(42, 46)
    DRAFT_MODEL_TPS, VERIFY_BATCH_SIZE, KV_CACHE_UTILIZATION, CUDA_GRAPH_ACTIVE = range(46, 50)
    DECODE_LATENCY_PER_TOKEN, V3_BLOCK_DEPTH, HOLO_FUTURE_SAFE, POWER_WATTS_NORM = range(50, 54)
    FLEET_HIT_RATE, FLEET_MISS_RATE, FLEET_EVICTION_RATE, FLEET_BLOCK_COUNT_NORM = range(54, 58)
    FLEET_WORKER_COUNT, FLEET_AVG_WORKER_LOAD, FLEET_MAX_WORKER_LOAD = range(58, 61)
    FLEET_PREFILL_QUEUE_DEPTH, FLEET_DECODE_QUEUE_DEPTH, FLEET_KV_OVERLAP_AVG = range(61, 64)
    FLEET_AMF_ROUTED_RATIO, FLEET_RESTORE_RATIO, FLEET_CROSS_NODE_XFERS = range(64, 67)
    FLEET_TIER_G1_PCT, FLEET_TIER_G2_PCT, FLEET_TIER_G3G4_PCT = range(67, 70)


def _f(v: Any, default: float = 0.0) -> float:
    try:
        x = float(v)
        return x if math.isfinite(x) else default
    except (TypeError, ValueError):
        return default


def _c01(x: float) -> float:
    return max(0.0, min(1.0, x))


def _ema(cur: float, new: float, alpha: float) -> float:
    return cur * (1.0 - alpha) + new * alpha


class StateCollector:
    """Builds the vector from an engine (``LLMEngine``: ``stat``, ``amf.stat``, ``bm``), an
    optional worker (``queue_status()``), an optional :class:`PowerSampler`, and decode
    steps reported through :meth:`record_decode_step`. :meth:`sample` computes one vector;
    :meth:`start` samples every ``interval_s`` on a thread and :meth:`vector` returns the
    latest (a copy)."""

    def __init__(self, engine=None, worker=None, power: Optional["PowerSampler"] = None, interval_s: float = 0.1,
                 tps_scale: float = 10000.0, latency_scale_ms: float = 200.0):
        self.engine, self.worker, self.power = engine, worker, power
        self.interval_s = max(0.01, interval_s)
        self.tps_scale, self.latency_scale_ms = tps_scale, latency_scale_ms
        self._v = np.zeros(WIDTH, np.float32)
        self._mu = threading.Lock()
        self._prev: Dict[str, float] = {}
        self._t_prev = time.monotonic()
        self._tps_hist: deque = deque(maxlen=50)
        self._acc = {"ema": 0.0, "var": 0.0, "depth": 0.0, "entropy": 0.5, "bad": 0.0, "lat": 0.0}
        self._streak = [0, 0]  # hits, misses in a row
        self._roi = 0.0
        self._roi_seen = False
        self._thread: Optional[threading.Thread] = None
        self._stop = threading.Event()

    # ------------------------------------------------------------------ inputs
    def record_decode_step(self, drafted: int, accepted: int, depth: int, entropy: float = 0.5,
                           latency_ms_per_token: float = 0.0) -> None:
        rate = accepted / drafted if drafted > 0 else 0.0
        with self._mu:
            a = self._acc
            d = rate - a["ema"]
            a["ema"] = _ema(a["ema"], rate, 0.2)
            a["var"] = _ema(a["var"], d * d, 0.2)
            a["depth"], a["entropy"] = float(depth), _ema(a["entropy"], _c01(entropy), 0.2)
            a["bad"] = a["bad"] + 1 if rate < 0.5 else 0.0
            if latency_ms_per_token > 0:
                a["lat"] = _ema(a["lat"] or latency_ms_per_token, latency_ms_per_token, 0.2)

    def record_lookup(self, hit: bool, savings_ms: float = 0.0, restore_ms: float = 0.0) -> None:
        with self._mu:
            self._streak = [self._streak[0] + 1, 0] if hit else [0, self._streak[1] + 1]
            if hit and savings_ms > 0:
                x = (savings_ms - restore_ms) / max(savings_ms, 1e-3)  # net fraction of the prefill saved
                self._roi = x if not self._roi_seen else _ema(self._roi, x, 0.1)
                self._roi_seen = True

    # ------------------------------------------------------------------ sampling
    def _delta(self, key: str, now: float) -> float:
        d = now - self._prev.get(key, now)
        self._prev[key] = now
        return d

    def sample(self) -> np.ndarray:
        v = np.zeros(WIDTH, np.float32)
        t = time.monotonic()
        dt = max(1e-3, t - self._t_prev)
        self._t_prev = t
        eng = self.engine
        with self._mu:
            if eng is not None:
                st = dict(getattr(eng, "stat", {}) or {})
                amf = dict(getattr(getattr(eng, "amf", None), "stat", {}) or {})
                hits = sum(_f(amf.get(k)) for k in amf if k.startswith("hits_"))
                misses = _f(amf.get("misses"))
                dh, dm = self._delta("hits", hits), self._delta("misses", misses)
                v[Slot.HIT_DELTA], v[Slot.MISS_DELTA] = dh, dm
                v[Slot.HIT_RATE] = hits / (hits + misses) if hits + misses else 0.0
                v[Slot.TOKENS_SAVED_DELTA] = self._delta("restored", _f(st.get("restored_tokens"))) / 1e5
                v[Slot.RESTORE_MS_AVG] = _c01(_f(amf.get("restore_ms")) / max(hits, 1.0) / self.latency_scale_ms)
                v[Slot.ADMISSION_RATE] = self._delta("captures", _f(amf.get("captures"))) / dt
                v[Slot.FAILURE_RATE] = self._delta("capfail", _f(amf.get("capture_failures"))) / dt
                v[Slot.REQUEST_RATE] = (dh + dm) / dt
                toks = self._delta("decode", _f(st.get("decode_tokens"))) + self._delta("prefill",
                                                                                       _f(st.get("prefill_tokens")))
                tps = toks / dt
                self._tps_hist.append(tps)
                v[Slot.INSTANT_TPS_NORM] = _c01(tps / self.tps_scale)
                v[Slot.ROLLING_TPS_NORM] = _c01(float(np.mean(self._tps_hist)) / self.tps_scale)
                v[Slot.TPS_CURRENT] = v[Slot.INSTANT_TPS_NORM]
                if len(self._tps_hist) > 1:
                    v[Slot.TPS_DELTA] = (self._tps_hist[-1] - self._tps_hist[-2]) / self.tps_scale
                bm = getattr(eng, "bm", None)
                total = _f(getattr(bm, "num_blocks", 0))
                free = _f(getattr(bm, "num_free", lambda: 0)() if callable(getattr(bm, "num_free", None))
                          else getattr(bm, "num_free", 0))
                if total > 0:
                    v[Slot.KV_CACHE_UTILIZATION] = _c01(1.0 - free / total)
                    v[Slot.MEMORY_PRESSURE] = v[Slot.KV_CACHE_UTILIZATION]
                v[Slot.CUDA_GRAPH_ACTIVE] = 1.0 if getattr(eng, "_graphs", None) is not None else 0.0
            v[Slot.HIT_STREAK_NORM] = _c01(self._streak[0] / 10.0)
            v[Slot.MISS_STREAK_NORM] = _c01(self._streak[1] / 10.0)
            v[Slot.ROI_EMA_NORM] = max(-1.0, min(1.0, self._roi / 10.0))
            a = self._acc
            v[Slot.ACCEPTANCE_EMA], v[Slot.ACCEPTANCE_VARIANCE] = a["ema"], a["var"]
            v[Slot.CURRENT_SPEC_DEPTH] = a["depth"] / 16.0
            v[Slot.ENTROPY_EMA] = a["entropy"]
            v[Slot.SPEC_BAD_STREAK] = _c01(a["bad"] / 10.0)
            v[Slot.SPEC_PROFIT_RATIO] = a["ema"] * a["depth"] / max(1.0, a["depth"] + 1.0)
            v[Slot.DECODE_LATENCY_PER_TOKEN] = _c01(a["lat"] / self.latency_scale_ms)
            v[Slot.DECODE_LATENCY_NORM] = v[Slot.DECODE_LATENCY_PER_TOKEN]
        if self.worker is not None:
            qs = self.worker.queue_status()
            dep = qs.get("depths", {})
            v[Slot.HIT_QUEUE_NORM] = _c01((dep.get("HIT", 0) + dep.get("SPEC_HIT", 0)) / 64.0)
            v[Slot.MISS_QUEUE_NORM] = _c01((dep.get("MISS", 0) + dep.get("SPEC_MISS", 0)) / 64.0)
        if self.power is not None:
            p = self.power.read()
            if p["limit_w"] > 0:
                v[Slot.POWER_WATTS_NORM] = _c01(p["watts"] / p["limit_w"])
        with self._mu:
            self._v = v
        return v.copy()

    def vector(self) -> np.ndarray:
        with self._mu:
            return self._v.copy()

    def start(self) -> "StateCollector":
        def loop():
            while not self._stop.wait(self.interval_s):
                try:
                    self.sample()
                except Exception:  # a failed sample keeps the previous vector
                    pass

        self._thread = threading.Thread(target=loop, daemon=True, name="policy-state")
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2.0)


class PowerSampler:
    """Board power of one GPU through NVML, averaged over the last ``window_s``. Read-only."""

    def __init__(self, device_index: int = 0, nvml=None, window_s: float = 1.0,
                 clock: Callable[[], float] = time.monotonic):
        if nvml is None:
            import pynvml as nvml  # nvidia-ml-py
        self.nvml, self.clock, self.window_s = nvml, clock, window_s
        nvml.nvmlInit()
        self.h = nvml.nvmlDeviceGetHandleByIndex(device_index)
        self._samples: deque = deque()

    def read(self) -> Dict[str, float]:
        now = self.clock()
        w = self.nvml.nvmlDeviceGetPowerUsage(self.h) / 1000.0
        try:
            lim = self.nvml.nvmlDeviceGetEnforcedPowerLimit(self.h) / 1000.0
        except Exception:
            lim = 0.0
        self._samples.append((now, w))
        while self._samples and now - self._samples[0][0] > self.window_s:
            self._samples.popleft()
        avg = sum(s[1] for s in self._samples) / len(self._samples)
        return {"watts": w, "avg_watts": avg, "limit_w": lim}

    def close(self) -> None:
        try:
            self.nvml.nvmlShutdown()
        except Exception:
            pass
