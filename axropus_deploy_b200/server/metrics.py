"""Prometheus metrics with the reference's names (axropus/metrics.py:1-60); no-op
stubs when prometheus_client is unavailable."""
from __future__ import annotations

from typing import Any, Dict

try:  # pragma: no cover - prometheus_client is installed here
    from prometheus_client import CollectorRegistry, Counter, Gauge, Summary, generate_latest
    _HAVE = True
except Exception:  # pragma: no cover
    _HAVE = False


class _Noop:
    def labels(self, *a, **k):
        return self

    def inc(self, *a, **k):
        pass

    def set(self, *a, **k):
        pass

    def observe(self, *a, **k):
        pass


class MetricRegistry:
    def __init__(self, enabled: bool = True):
        self.enabled = enabled and _HAVE
        if not self.enabled:
            n = _Noop()
            self.cache_hits = self.cache_latency = self.prefixes = self.pool_bytes = n
            self.evictions = self.compression = self.kernel_latency = self.tokens_saved = n
            self.cost_saved = self.miss_reason = self.requests = self.ttft = n
            self.registry = None
            return
        r = self.registry = CollectorRegistry()
        self.cache_hits = Counter("axropus_cache_hits_total", "lookups served per tier", ["tier"], registry=r)
        self.cache_latency = Summary("axropus_cache_latency_ms", "lookup latency per tier", ["tier"], registry=r)
        self.prefixes = Gauge("axropus_pool_prefixes_resident", "prefixes resident in G1", registry=r)
        self.pool_bytes = Gauge("axropus_pool_bytes_used", "bytes used in G1", registry=r)
        self.evictions = Counter("axropus_pool_evictions_total", "G1 evictions", registry=r)
        self.compression = Gauge("axropus_compression_ratio", "stored/fp16 bytes", ["codec"], registry=r)
        self.kernel_latency = Summary("axropus_kernel_latency_us", "kernel latency", ["kernel"], registry=r)
        self.tokens_saved = Counter("axropus_tokens_saved_total", "prefill tokens skipped by restores", registry=r)
        self.cost_saved = Counter("axropus_compute_cost_saved_usd", "estimated compute cost saved", registry=r)
        self.miss_reason = Counter("axropus_miss_reason_total", "misses by reason", ["reason"], registry=r)
        self.requests = Counter("axropus_requests_total", "requests served", ["endpoint"], registry=r)
        self.ttft = Summary("axropus_ttft_ms", "time to first token", ["tier"], registry=r)
        self._last_evictions = 0

    def observe_request(self, tier: str, ttft_ms: float, restored_tokens: int, gpu_hour_usd: float = 3.0,
                        prefill_tok_per_s: float = 50000.0) -> None:
        self.cache_hits.labels(tier=tier).inc()
        self.ttft.labels(tier=tier).observe(ttft_ms)
        if restored_tokens:
            self.tokens_saved.inc(restored_tokens)
            self.cost_saved.inc(restored_tokens / prefill_tok_per_s / 3600.0 * gpu_hour_usd)

    def update_pool(self, stats: Dict[str, Any]) -> None:
        self.prefixes.set(stats.get("num_prefixes", 0))
        self.pool_bytes.set(stats.get("used_bytes", 0))
        ev = stats.get("evictions", 0)
        if ev > self._last_evictions:
            self.evictions.inc(ev - self._last_evictions)
            self._last_evictions = ev

    def render(self) -> bytes:
        return generate_latest(self.registry) if self.enabled else b""
