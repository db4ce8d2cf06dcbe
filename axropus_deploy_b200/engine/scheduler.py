"""Admission policy of the engine: which waiting request goes next, and how many prefill
tokens a step may take while requests are decoding.

Score (highest first), per waiting request:
``(starved, replay, -priority, lane_bias, short)`` where ``starved`` is 1 after
``KORITH_VLLM_STARVATION_S`` of waiting, ``replay`` is 1.06 when its prefix is held by the
AMF tiers or the live prefix cache (cheap to admit: restore, not prefill), ``lane_bias``
comes from ``KORITH_VLLM_LANE_BIAS_{SPEC_HIT,HIT,SPEC_MISS,MISS}`` and ``short`` prefers
fewer tokens to prefill (the prefill penalty of long cold prompts). The order is stable, so
equal scores stay first-come first-served.

Budget: when the share of decoding requests in the batch reaches
``KORITH_VLLM_DECODE_RATIO_THRESHOLD``, a step's prefill budget is scaled by
``KORITH_VLLM_BUDGET_SCALE_DECODE`` (never below ``KORITH_VLLM_MIN_SCHEDULED_TOKENS``)
so running decodes keep a short step time -- except when the head of the queue is a hit and
``KORITH_VLLM_DECODE_FULL_BUDGET_ON_HIT`` is set. ``KORITH_VLLM_DECODE_FIRST=0`` turns the
policy off (plain first-come first-served, full budget).

Trace: with ``KORITH_VLLM_SCHED_TRACE_PATH`` and ``KORITH_VLLM_SCHED_TRACE_EVERY=N``, every
N-th admission round appends one JSON line (queue length, requests decoding, prefill budget,
whether the head of the queue is a hit, how many were admitted, how many waiting requests
are held by a cache tier).

Reference: korith_vllm_ext/decode_scheduler.py:89-147 (the knobs and their defaults) and
:326-377 (the request score), a vLLM scheduler subclass there; here the engine's own
admission loop consults it.
"""
from __future__ import annotations

import json
import os
import time
from typing import List


def _f(name: str, default: float, lo: float, hi: float) -> float:
    try:
        v = float(os.environ.get(name, default))
    except ValueError:
        v = default
    return max(lo, min(hi, v))


def _b(name: str, default: bool) -> bool:
    v = os.environ.get(name)
    return default if v is None else v.strip().lower() in ("1", "true", "yes", "on")


class AdmissionPolicy:
    def __init__(self):
        self.enabled = _b("KORITH_VLLM_DECODE_FIRST", True)
        self.adaptive = _b("KORITH_VLLM_ADAPTIVE_BUDGET", True)
        self.scale_decode = _f("KORITH_VLLM_BUDGET_SCALE_DECODE", 0.75, 0.25, 1.0)
        self.ratio_threshold = _f("KORITH_VLLM_DECODE_RATIO_THRESHOLD", 0.6, 0.0, 1.0)
        self.min_tokens = int(_f("KORITH_VLLM_MIN_SCHEDULED_TOKENS", 128, 1, 1 << 30))
        self.starvation_s = _f("KORITH_VLLM_STARVATION_S", 0.75, 0.0, 1e9)
        self.full_on_hit = _b("KORITH_VLLM_DECODE_FULL_BUDGET_ON_HIT", True)
        self.lane_bias = {lane: _f(f"KORITH_VLLM_LANE_BIAS_{lane}", d, 0.1, 10.0)
                          for lane, d in (("SPEC_HIT", 1.25), ("HIT", 1.1), ("SPEC_MISS", 0.95), ("MISS", 1.0))}
        self.trace_path = os.environ.get("KORITH_VLLM_SCHED_TRACE_PATH", "")
        self.trace_every = int(_f("KORITH_VLLM_SCHED_TRACE_EVERY", 0, 0, 1 << 30))
        self.rounds = 0

    def note(self, **fields) -> None:
        """Count an admission round; every ``trace_every``-th one goes to the trace file."""
        self.rounds += 1
        if self.trace_path and self.trace_every > 0 and self.rounds % self.trace_every == 0:
            with open(self.trace_path, "a") as f:
                f.write(json.dumps({"ts": time.time(), "round": self.rounds, "enabled": self.enabled, **fields}) + "\n")

    def order(self, waiting: List, held, spec: bool = False, now: float = None) -> List:
        """Waiting requests in admission order; ``held(r)`` says whether r's prefix is
        held by a cache tier (cached on the request)."""
        if not self.enabled or len(waiting) < 2:
            return waiting
        t = time.perf_counter() if now is None else now

        def score(r):
            hit = r.__dict__.setdefault("_held", held(r))
            lane = ("SPEC_" if spec else "") + ("HIT" if hit else "MISS")
            starved = 1.0 if t - r.t_arrival >= self.starvation_s else 0.0
            return (starved, 1.06 if hit else 1.0, -getattr(r.params, "priority", 0), self.lane_bias[lane],
                    -len(r.prompt) if not hit else 0)

        return sorted(waiting, key=score, reverse=True)

    def budget(self, max_tokens: int, decoding: int, max_batch: int, head_is_hit: bool) -> int:
        if not (self.enabled and self.adaptive) or max_batch <= 0:
            return max_tokens
        if decoding / max_batch < self.ratio_threshold or (head_is_hit and self.full_on_hit):
            return max_tokens
        return max(self.min_tokens, int(max_tokens * self.scale_decode))
