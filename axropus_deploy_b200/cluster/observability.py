"""Control-plane observability: an in-process counter/gauge registry rendered as
Prometheus text, JSON log lines, and the per-job artifact store.

* :class:`MetricsRegistry` -- thread-safe counters and gauges keyed by name + labels.
  Organisation ids are a high-cardinality label; ``KORITH_METRICS_ORG_LABEL_MODE``
  chooses how they are exported: ``bounded`` (default: the first
  ``KORITH_METRICS_MAX_ORG_LABELS`` orgs get stable aliases, the rest ``other``; an
  optional ``KORITH_METRICS_ORG_ALLOWLIST``), ``hash`` (a short digest) or ``raw``.
* :func:`emit_log` -- one JSON object per line (timestamp, service, event, fields) on
  stdout and, optionally, appended to a job's log file.
* :class:`ArtifactStore` -- a directory per (org, job) holding ``metrics.json``,
  ``events.jsonl``, ``output.txt``, ``run.log`` and the KV snapshot of the run.

Reference: platform/observability/metrics.py:9-92, platform/observability/platform_logging.py:14-40,
platform/artifacts/store.py (directory layout).
"""
from __future__ import annotations

import hashlib
import json
import os
import threading
from datetime import datetime, timezone
from pathlib import Path
from typing import Any, Dict, Optional


def utc_now() -> str:
    return datetime.now(timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ")


class MetricsRegistry:
    def __init__(self, org_label_mode: Optional[str] = None, max_org_labels: Optional[int] = None,
                 org_allowlist: Optional[set] = None):
        self._mu = threading.Lock()
        self.counters: Dict[str, float] = {}
        self.gauges: Dict[str, float] = {}
        self.mode = (org_label_mode or os.environ.get("KORITH_METRICS_ORG_LABEL_MODE", "bounded")).strip().lower()
        env_max = os.environ.get("KORITH_METRICS_MAX_ORG_LABELS", "200").strip()
        self.max_orgs = max_org_labels or (max(1, int(env_max)) if env_max.isdigit() else 200)
        env_allow = {x.strip() for x in os.environ.get("KORITH_METRICS_ORG_ALLOWLIST", "").split(",") if x.strip()}
        self.allow = org_allowlist if org_allowlist is not None else env_allow
        self._alias: Dict[str, str] = {}

    def _org(self, org: str) -> str:
        if self.mode == "raw":
            return org
        if self.mode == "hash":
            return "org_" + hashlib.sha1(org.encode("utf-8")).hexdigest()[:12]
        if self.allow and org not in self.allow:
            return "other"
        if org not in self._alias:
            if len(self._alias) >= self.max_orgs:
                return "other"
            self._alias[org] = f"org_{len(self._alias) + 1:04d}"
        return self._alias[org]

    def _key(self, name: str, labels: Optional[Dict[str, Any]]) -> str:
        if not labels:
            return name
        items = sorted((str(k), self._org(str(v)) if k == "org_id" else str(v)) for k, v in labels.items())
        inner = ",".join(f'{k}="{v}"' for k, v in items)
        return f"{name}{{{inner}}}"

    def inc(self, name: str, value: float = 1.0, labels: Optional[Dict[str, Any]] = None) -> None:
        with self._mu:
            k = self._key(name, labels)
            self.counters[k] = self.counters.get(k, 0.0) + float(value)

    def set_gauge(self, name: str, value: float, labels: Optional[Dict[str, Any]] = None) -> None:
        with self._mu:
            self.gauges[self._key(name, labels)] = float(value)

    def get_counter(self, name: str, labels: Optional[Dict[str, Any]] = None) -> float:
        with self._mu:
            return self.counters.get(self._key(name, labels), 0.0)

    def get_gauge(self, name: str, labels: Optional[Dict[str, Any]] = None) -> float:
        with self._mu:
            return self.gauges.get(self._key(name, labels), 0.0)

    def snapshot(self) -> Dict[str, Dict[str, float]]:
        with self._mu:
            return {"counters": dict(self.counters), "gauges": dict(self.gauges)}

    def render_prometheus(self) -> str:
        with self._mu:
            lines, typed = [], set()
            for kind, table in (("counter", self.counters), ("gauge", self.gauges)):
                for k in sorted(table):
                    base = k.split("{", 1)[0]
                    if base not in typed:
                        lines.append(f"# TYPE {base} {kind}")
                        typed.add(base)
                    lines.append(f"{k} {table[k]:g}")
            return "\n".join(lines) + ("\n" if lines else "")


GLOBAL_METRICS = MetricsRegistry()


def emit_log(service: str, event: str, fields: Dict[str, Any], artifact_log: Optional[Path] = None,
             echo: bool = True) -> Dict[str, Any]:
    payload = {"timestamp": utc_now(), "service": service, "event": event, **fields}
    line = json.dumps(payload, ensure_ascii=False, default=str)
    if echo:
        print(line, flush=True)
    if artifact_log is not None:
        artifact_log.parent.mkdir(parents=True, exist_ok=True)
        with artifact_log.open("a", encoding="utf-8") as f:
            f.write(line + "\n")
    return payload


def error_fields(error: BaseException, replay_related: bool = False) -> Dict[str, Any]:
    return {"error_type": type(error).__name__, "error": str(error), "replay_related": replay_related}


class ArtifactStore:
    """Local artifact directories: ``<base>/<org>/<job>/{metrics.json, events.jsonl,
    output.txt, run.log, kv_snapshot.amfk, engine_metrics.json, engine_events.jsonl}``."""

    def __init__(self, base_dir):
        self.base = Path(base_dir)
        self.base.mkdir(parents=True, exist_ok=True)

    def init_job(self, job_id: str, org_id: str = "default") -> Dict[str, Path]:
        d = self.base / org_id / job_id
        d.mkdir(parents=True, exist_ok=True)
        return {"job_dir": d, "metrics": d / "metrics.json", "events": d / "events.jsonl", "output": d / "output.txt",
                "log": d / "run.log", "snapshot": d / "kv_snapshot.amfk", "engine_metrics": d / "engine_metrics.json",
                "engine_events": d / "engine_events.jsonl"}

    @staticmethod
    def append_event(events_path: Path, event: Any) -> None:
        with Path(events_path).open("a", encoding="utf-8") as f:
            f.write((event if isinstance(event, str) else json.dumps(event, ensure_ascii=False, default=str)) + "\n")

    @staticmethod
    def write_json(path: Path, obj: Any) -> None:
        Path(path).write_text(json.dumps(obj, indent=2, ensure_ascii=False, default=str), encoding="utf-8")

    @staticmethod
    def read_events(path: Path) -> list:
        out = []
        p = Path(path)
        if not p.exists():
            return out
        for line in p.read_text(encoding="utf-8").splitlines():
            line = line.strip()
            if line:
                try:
                    out.append(json.loads(line))
                except ValueError:
                    out.append({"raw": line})
        return out
