"""Node-side agent of the hosted backend: registers a freshly deployed serving node and
reports its usage.

Started beside ``axropus serve`` by the backend's SSH deployment (or by hand):

    python -m axropus_deploy_b200.saas.agent --backend https://backend --deployment-id 7 \\
        --api-key ax-... --port 8000 [--public-url http://host:8000]

1. waits for the local server's ``/healthz``;
2. registers ``public_url`` with ``POST /api/deploy/{id}/register`` (retried);
3. every ``interval`` seconds reads the server's ``/stats`` (engine counters) and posts the
   increments as one usage report to ``/api/metrics``: tokens processed (prefill +
   decode), prefix tokens skipped (restored + reused from the local prefix cache), decode
   tokens accelerated (accepted speculative drafts), AMF hit rate, speculative acceptance,
   effective throughput and the share of prefill compute saved. Only these numbers leave
   the node; no prompt or output does.

Reference counterpart: platform/runtime/gateway_agent.py:88-176 (register, metrics loop).
"""
from __future__ import annotations

import argparse
import json
import socket
import threading
import time
import urllib.request
from datetime import datetime, timezone
from typing import Any, Callable, Dict, Optional


def _post_json(url: str, payload: Dict[str, Any], timeout: float = 10.0) -> Dict[str, Any]:
    req = urllib.request.Request(url, json.dumps(payload).encode(), {"Content-Type": "application/json"})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.loads(r.read() or b"{}")


def _get_json(url: str, headers: Optional[Dict[str, str]] = None, timeout: float = 5.0) -> Dict[str, Any]:
    req = urllib.request.Request(url, headers=headers or {})
    with urllib.request.urlopen(req, timeout=timeout) as r:
        return json.loads(r.read() or b"{}")


def _host_ip() -> str:
    s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
    try:
        s.connect(("10.255.255.255", 1))  # no packet is sent: picks the outbound interface
        return s.getsockname()[0]
    except OSError:
        return "127.0.0.1"
    finally:
        s.close()


def usage_report(prev: Dict[str, Any], cur: Dict[str, Any], interval_s: float, gpu_count: int) -> Dict[str, Any]:
    """Usage fields of one report from two engine ``stats()`` snapshots (increments)."""
    def d(key, sub=None):
        a = (cur.get(sub) or {}) if sub else cur
        b = (prev.get(sub) or {}) if sub else prev
        return max(0.0, float(a.get(key, 0) or 0) - float(b.get(key, 0) or 0))

    prefill, decode = d("prefill_tokens"), d("decode_tokens")
    skipped = d("restored_tokens") + d("local_cached_tokens")
    cold = d("cold_prefill_tokens")
    drafted, accepted = d("drafted", "spec"), d("accepted", "spec")
    lookups, misses = d("lookups", "amf"), d("misses", "amf")
    hits = max(0.0, lookups - misses)  # hits of every tier (G1 raw / pool, CPU, NVMe, disk)
    processed = prefill + decode
    saved = skipped / (skipped + cold) if skipped + cold > 0 else 0.0
    return {
        "interval_seconds": int(round(interval_s)),
        "tokens_processed": int(processed),
        "prefix_skipped": int(skipped),
        "decode_accelerated": int(accepted),
        "amf_hit_rate": round(hits / (hits + misses), 6) if hits + misses > 0 else 0.0,
        "spec_acceptance_rate": round(accepted / drafted, 6) if drafted > 0 else 0.0,
        "effective_tps": round(processed / interval_s, 3) if interval_s > 0 else 0.0,
        "baseline_tps": round((processed - skipped) / interval_s, 3) if interval_s > 0 else 0.0,
        "compute_saved_pct": round(min(1.0, saved), 6),
        "gpu_count": int(gpu_count),
        "heartbeat": 1,
    }


class Agent:
    def __init__(self, backend: str, api_key: str, deployment_id: int, port: int = 8000,
                 public_url: Optional[str] = None, interval_s: float = 60.0, gpu_count: int = 1,
                 model_family: str = "llama3", post_json: Callable = _post_json, get_json: Callable = _get_json,
                 clock: Callable[[], float] = time.monotonic):
        self.backend = backend.rstrip("/")
        self.api_key, self.dep, self.port = api_key, int(deployment_id), int(port)
        self.public_url = public_url or f"http://{_host_ip()}:{self.port}"
        self.local = f"http://127.0.0.1:{self.port}"
        self.interval_s, self.gpu_count, self.family = float(interval_s), int(gpu_count), model_family
        self.post_json, self.get_json, self.clock = post_json, get_json, clock
        self._stop = threading.Event()
        self._prev: Optional[Dict[str, Any]] = None
        self._t_prev = 0.0
        self.reports = 0

    def wait_healthy(self, timeout_s: float = 600.0) -> bool:
        end = self.clock() + timeout_s
        while not self._stop.is_set():
            try:
                if self.get_json(self.local + "/healthz").get("ok"):
                    return True
            except Exception:
                pass
            if self.clock() >= end:
                return False
            self._stop.wait(1.0)
        return False

    def register(self, attempts: int = 3) -> bool:
        for i in range(attempts):
            try:
                self.post_json(f"{self.backend}/api/deploy/{self.dep}/register",
                               {"api_key": self.api_key, "inference_url": self.public_url})
                return True
            except Exception:
                self._stop.wait(min(10.0, 2.0 ** i))
        return False

    def report_once(self) -> Optional[Dict[str, Any]]:
        """One usage report (None on the first call, which only takes the baseline)."""
        cur = self.get_json(self.local + "/stats", {"Authorization": "Bearer " + self.api_key})
        now = self.clock()
        if self._prev is None:
            self._prev, self._t_prev = cur, now
            return None
        body = usage_report(self._prev, cur, now - self._t_prev, self.gpu_count)
        body.update({"api_key": self.api_key, "model_family": self.family,
                     "timestamp": datetime.now(timezone.utc).isoformat(timespec="seconds")})
        self.post_json(self.backend + "/api/metrics", body)
        self._prev, self._t_prev = cur, now
        self.reports += 1
        return body

    def run(self) -> None:
        if not self.wait_healthy() or not self.register():
            return
        while not self._stop.is_set():
            try:
                self.report_once()
            except Exception:
                pass  # the backend or the server is briefly away: try again next interval
            self._stop.wait(self.interval_s)

    def stop(self) -> None:
        self._stop.set()


def main() -> None:
    ap = argparse.ArgumentParser(description="register a serving node with the hosted backend and report usage")
    ap.add_argument("--backend", required=True)
    ap.add_argument("--deployment-id", type=int, required=True)
    ap.add_argument("--api-key", required=True)
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--public-url", default=None)
    ap.add_argument("--interval", type=float, default=60.0)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--model-family", default="llama3")
    a = ap.parse_args()
    Agent(a.backend, a.api_key, a.deployment_id, a.port, a.public_url, a.interval, a.gpus, a.model_family).run()


if __name__ == "__main__":
    main()
