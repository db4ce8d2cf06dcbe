"""AMF trace lines and engine events.

The reference's engine prints one line per AMF decision on stderr -- ``[AMF_KEY]``,
``[AMF_HIT]``, ``[AMF_MISS]``, ``[AMF_SKIP]``, ``[AMF_STATS]`` and a closing
``[KORITH_RUN_SUMMARY]`` (core/engine.cpp:1865, :2718, :2896-2935, :3010, :3096) -- and the
platform parses them, so the field names and order are kept. Lines are written when
``KORITH_AMF_TRACE=1`` (or ``EngineConfig.trace``) to stderr or ``KORITH_AMF_TRACE_PATH``.
Engine events go as JSON lines to ``KORITH_ENGINE_EVENTS_PATH`` and the run's metrics as
JSON to ``KORITH_ENGINE_METRICS_PATH`` (core/engine.cpp:427-441, :2102-2107).
"""
from __future__ import annotations

import json
import os
import sys
import time
from typing import IO, Optional


class AmfTrace:
    def __init__(self, enabled: Optional[bool] = None, stream: Optional[IO] = None):
        env = os.environ.get("KORITH_AMF_TRACE", "0").lower() in ("1", "true", "yes", "on")
        self.enabled = env if enabled is None else enabled
        path = os.environ.get("KORITH_AMF_TRACE_PATH")
        self.stream = stream or (open(path, "a", buffering=1) if (path and self.enabled) else sys.stderr)
        self.events_path = os.environ.get("KORITH_ENGINE_EVENTS_PATH")
        self.metrics_path = os.environ.get("KORITH_ENGINE_METRICS_PATH")
        # running cold-prefill rate, to express a hit as prefill time saved
        self.prefill_tok = 0
        self.prefill_ms = 0.0
        self.n = {"hits": 0, "misses": 0, "skipped_tokens": 0, "prompt_tokens": 0, "saved_ms": 0.0, "roi_sum": 0.0,
                  "tokens_generated": 0, "t0": time.perf_counter()}

    def _line(self, s: str) -> None:
        if self.enabled:
            self.stream.write(s + "\n")

    def event(self, kind: str, **fields) -> None:
        if self.events_path:
            with open(self.events_path, "a") as f:
                f.write(json.dumps({"type": kind, "ts": time.time(), **fields}) + "\n")

    def prefill_rate(self) -> float:
        return self.prefill_tok / (self.prefill_ms * 1e-3) if self.prefill_ms > 0 else 0.0

    def note_prefill(self, tokens: int, ms: float) -> None:
        self.prefill_tok += tokens
        self.prefill_ms += ms

    def key(self, result: str, model_hash: int, tenant_hash: int, prompt_hash: int, n_ctx: int, n_batch: int,
            rope_base: int = 0, rope_scale: int = 0, sampling_hash: int = 0, seed: int = 0) -> None:
        self._line(f"[AMF_KEY] result={result} model_hash={model_hash:x} tenant_hash={tenant_hash:x} "
                   f"prompt_hash={prompt_hash:x} n_ctx={n_ctx} n_batch={n_batch} rope_base=0x{rope_base:08x} "
                   f"rope_scale=0x{rope_scale:08x} sampling_hash={sampling_hash:x} seed={seed:x}")

    def hit(self, prompt_tokens: int, prefix_tokens: int, skipped_tokens: int, restore_ms: float, tier: str) -> None:
        rate = self.prefill_rate()
        baseline_ms = skipped_tokens / rate * 1e3 if rate > 0 else 0.0
        saved_ms = max(0.0, baseline_ms - restore_ms)
        roi = saved_ms / restore_ms if restore_ms > 0 else 0.0
        skip_ratio = skipped_tokens / prompt_tokens if prompt_tokens else 0.0
        self.n["hits"] += 1
        self.n["skipped_tokens"] += skipped_tokens
        self.n["prompt_tokens"] += prompt_tokens
        self.n["saved_ms"] += saved_ms
        self.n["roi_sum"] += roi
        self._line(f"[AMF_SKIP] prompt_tokens={prompt_tokens} skipped_tokens={skipped_tokens} "
                   f"skip_ratio={skip_ratio:.3f} restore_ms={restore_ms:.2f} saved_ms={saved_ms:.2f} roi={roi:.2f}")
        self._line(f"[AMF_HIT] prefix_tokens={prefix_tokens} skipped_tokens={skipped_tokens} "
                   f"baseline_ms={baseline_ms:.2f} restore_ms={restore_ms:.2f} saved_ms={saved_ms:.2f} roi={roi:.2f}")
        self.event("amf_hit", tier=tier, prefix_tokens=prefix_tokens, skipped_tokens=skipped_tokens,
                   restore_ms=restore_ms, saved_ms=saved_ms)

    def miss(self, reason: str, prompt_ms: float, tokens: int) -> None:
        self.n["misses"] += 1
        self.n["prompt_tokens"] += tokens
        tps = tokens / (prompt_ms * 1e-3) if prompt_ms > 0 else 0.0
        self._line(f"[AMF_MISS] reason={reason} prompt_ms={prompt_ms:.2f} tokens={tokens} base_prompt_tps={tps:.2f}")
        self.event("amf_miss", reason=reason, tokens=tokens, prompt_ms=prompt_ms)

    def stats(self, s: dict) -> None:
        self._line("[AMF_STATS] " + " ".join(f"{k}={int(v) if isinstance(v, float) else v}" for k, v in s.items()))

    def summary(self, tokens_generated: int, fallback_used: bool = False) -> dict:
        el = time.perf_counter() - self.n["t0"]
        n = self.n
        out = {"tokens_generated": tokens_generated, "avg_tps": tokens_generated / el if el > 0 else 0.0,
               "amf_hit": int(n["hits"] > 0),
               "avg_skip_ratio": min(1.0, n["skipped_tokens"] / n["prompt_tokens"]) if n["prompt_tokens"] else 0.0,
               "avg_roi": n["roi_sum"] / n["hits"] if n["hits"] else 0.0, "fallback_used": int(fallback_used)}
        self._line(f"[KORITH_RUN_SUMMARY] tokens_generated={out['tokens_generated']} avg_tps={out['avg_tps']:.2f} "
                   f"amf_hit={out['amf_hit']} avg_skip_ratio={out['avg_skip_ratio']:.3f} "
                   f"avg_roi={out['avg_roi']:.2f} fallback_used={out['fallback_used']}")
        if self.metrics_path:
            with open(self.metrics_path, "w") as f:
                json.dump(dict(out, hits=n["hits"], misses=n["misses"], saved_ms=n["saved_ms"]), f)
        return out
