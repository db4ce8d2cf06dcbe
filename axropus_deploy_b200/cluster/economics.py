"""Savings accounting: what the AMF restores and speculative decoding saved, in GPU time
and money, per run, per tenant and against savings targets.

A run's ``metrics.json`` (written by :class:`~.worker.ClusterWorker`) carries
``perf`` (``total_ms``, ``prefill_ms``, ``decode_ms``), ``amf`` (``decision`` hit/miss,
``saved_ms`` = the cold-prefill time of the restored tokens minus the restore time) and
``spec`` (``saved_ms``). When a ``savings`` block lists ``prefill_saved_ms``,
``spec_saved_ms`` and ``kernels_saved_ms`` it is taken as is.

* :func:`extract_savings_components` / :func:`estimate_savings` -- one run;
* :class:`TenantMeter` -- running totals of a tenant (hit rate, saved vs served time,
  cost at a GPU-hour price);
* :func:`target_report` -- over the latest run of each ledger job: achieved savings %
  against a list of targets and the extra time each unmet target still needs;
* :func:`write_report` -- JSON, Markdown or a one-page PDF (written directly: a text page
  in the PDF 1.4 object syntax, no library).

Reference: platform/economics/model.py:13-100, tenant_meter.py:22-100, targets.py:48-160,
report.py:14-61.
"""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, Iterable, List, Optional

from .observability import utc_now

MS_PER_HOUR = 3_600_000.0


def _f(v: Any) -> float:
    try:
        return float(v or 0.0)
    except (TypeError, ValueError):
        return 0.0


def extract_savings_components(metrics: Dict[str, Any]) -> Dict[str, float]:
    sav = metrics.get("savings") if isinstance(metrics.get("savings"), dict) else None
    if sav and all(k in sav for k in ("prefill_saved_ms", "spec_saved_ms", "kernels_saved_ms")):
        p, s, k = (max(0.0, _f(sav[x])) for x in ("prefill_saved_ms", "spec_saved_ms", "kernels_saved_ms"))
    else:
        amf = metrics.get("amf") or {}
        spec = metrics.get("spec") or {}
        ker = metrics.get("kernels") or {}
        p = max(0.0, _f(amf.get("saved_ms")))
        # kernel savings only count when the kernels ran and were compared like for like
        k = max(0.0, _f(ker.get("ms_saved"))) if ker.get("kernels_applied") and ker.get("comparable", True) else 0.0
        s = max(0.0, _f(spec.get("saved_ms")) - k)
    return {"prefill_saved_ms": p, "spec_saved_ms": s, "kernels_saved_ms": k, "total_saved_ms": p + s + k}


def estimate_savings(metrics: Dict[str, Any], gpu_hourly_cost: float) -> Dict[str, float]:
    c = extract_savings_components(metrics)
    total_ms = _f((metrics.get("perf") or {}).get("total_ms"))
    per_ms = max(0.0, gpu_hourly_cost) / MS_PER_HOUR
    return dict(c, saved_ms=c["total_saved_ms"], total_ms=total_ms, gpu_cost_per_ms=per_ms,
                cost_saved_usd=c["total_saved_ms"] * per_ms, cost_total_usd=total_ms * per_ms)


@dataclass
class TenantMeter:
    tenant_id: str
    total_requests: int = 0
    amf_hits: int = 0
    amf_misses: int = 0
    prefill_saved_ms: float = 0.0
    decode_ms: float = 0.0
    total_saved_ms: float = 0.0
    total_compute_ms: float = 0.0
    cache_entries: int = 0
    cache_bytes: int = 0

    def accumulate(self, metrics: Dict[str, Any]) -> None:
        self.total_requests += 1
        amf = metrics.get("amf") or {}
        perf = metrics.get("perf") or {}
        d = str(amf.get("decision", "")).lower()
        self.amf_hits += d == "hit"
        self.amf_misses += d == "miss"
        c = extract_savings_components(metrics)
        self.prefill_saved_ms += c["prefill_saved_ms"]
        self.total_saved_ms += c["total_saved_ms"]
        self.total_compute_ms += max(0.0, _f(perf.get("total_ms")))
        self.decode_ms += max(0.0, _f(perf.get("decode_ms")))
        self.cache_entries = max(self.cache_entries, int(_f(amf.get("cache_entries"))))
        self.cache_bytes = max(self.cache_bytes, int(_f(amf.get("cache_bytes"))))

    def summary(self, gpu_hourly_cost: float = 2.5, period_start: str = "", period_end: str = "") -> Dict[str, Any]:
        per_ms = max(0.0, gpu_hourly_cost) / MS_PER_HOUR
        base = self.total_compute_ms + self.total_saved_ms
        now = utc_now()
        return {"tenant_id": self.tenant_id, "period_start": period_start or now, "period_end": period_end or now,
                "total_requests": self.total_requests,
                "amf_hit_rate": self.amf_hits / max(1, self.amf_hits + self.amf_misses),
                "total_saved_ms": self.total_saved_ms, "total_compute_ms": self.total_compute_ms,
                "savings_pct": 100.0 * self.total_saved_ms / base if base > 0 else 0.0,
                "cost_saved_usd": self.total_saved_ms * per_ms, "cost_served_usd": self.total_compute_ms * per_ms,
                "cache_entries": self.cache_entries, "cache_bytes": self.cache_bytes}


def _latest_metrics(ledger, limit: int, org_id: Optional[str]) -> Iterable[Dict[str, Any]]:
    for job in ledger.list_jobs(limit, org_id=org_id):
        run = ledger.get_latest_run(job["job_id"])
        p = Path(run["metrics_path"]) if run and run.get("metrics_path") else None
        if p is None or not p.exists():
            continue
        try:
            yield json.loads(p.read_text(encoding="utf-8"))
        except ValueError:
            continue


def target_report(ledger, targets: List[float], org_id: Optional[str] = None, limit: int = 5000) -> Dict[str, Any]:
    """Achieved savings over the latest run of each job vs ``targets`` (fractions, e.g. 0.3)."""
    obs = pre = dec = other = pre_saved = dec_saved = 0.0
    n = 0
    for m in _latest_metrics(ledger, limit, org_id):
        perf = m.get("perf") or {}
        c = extract_savings_components(m)
        t, p, d = _f(perf.get("total_ms")), _f(perf.get("prefill_ms")), _f(perf.get("decode_ms"))
        n += 1
        obs += t
        pre += p
        dec += d
        other += max(0.0, t - p - d)
        pre_saved += c["prefill_saved_ms"]
        dec_saved += c["spec_saved_ms"] + c["kernels_saved_ms"]
    base = obs + pre_saved + dec_saved
    achieved = (pre_saved + dec_saved) / base if base > 0 else 0.0
    rows = []
    for tgt in targets:
        need_ms = max(0.0, tgt * base - (pre_saved + dec_saved))
        rows.append({"target_pct": 100.0 * tgt, "met": achieved >= tgt, "additional_saved_ms_needed": need_ms,
                     # the share of the remaining prefill that restores would have to remove
                     "prefill_share_needed": min(1.0, need_ms / pre) if pre > 0 else None})
    return {"runs": n, "observed_total_ms": obs, "baseline_total_ms": base, "prefill_ms": pre, "decode_ms": dec,
            "other_ms": other, "prefill_saved_ms": pre_saved, "decode_saved_ms": dec_saved,
            "achieved_pct": 100.0 * achieved, "targets": rows}


def _pdf_escape(s: str) -> str:
    return s.replace("\\", "\\\\").replace("(", "\\(").replace(")", "\\)")


def write_pdf(path: Path, lines: List[str]) -> None:
    """One text page (Helvetica 10 pt, up to ~60 lines) in PDF 1.4 object syntax."""
    body = ["BT /F1 10 Tf 50 800 Td 13 TL"] + [f"({_pdf_escape(l[:110])}) '" for l in lines[:60]] + ["ET"]
    stream = "\n".join(body).encode("latin-1", "replace")
    objs = [b"<< /Type /Catalog /Pages 2 0 R >>",
            b"<< /Type /Pages /Kids [3 0 R] /Count 1 >>",
            b"<< /Type /Page /Parent 2 0 R /MediaBox [0 0 595 842] /Contents 4 0 R "
            b"/Resources << /Font << /F1 5 0 R >> >> >>",
            b"<< /Length " + str(len(stream)).encode() + b" >>\nstream\n" + stream + b"\nendstream",
            b"<< /Type /Font /Subtype /Type1 /BaseFont /Helvetica >>"]
    out = bytearray(b"%PDF-1.4\n")
    offs = []
    for i, o in enumerate(objs, 1):
        offs.append(len(out))
        out += f"{i} 0 obj\n".encode() + o + b"\nendobj\n"
    xref = len(out)
    out += f"xref\n0 {len(objs) + 1}\n0000000000 65535 f \n".encode()
    for o in offs:
        out += f"{o:010d} 00000 n \n".encode()
    out += f"trailer\n<< /Size {len(objs) + 1} /Root 1 0 R >>\nstartxref\n{xref}\n%%EOF\n".encode()
    Path(path).write_bytes(bytes(out))


def write_report(ledger, out_path, gpu_hourly_cost: float = 2.5, org_id: Optional[str] = None,
                 targets: Optional[List[float]] = None) -> Dict[str, Any]:
    """Savings report over the ledger; the file type follows ``out_path``'s suffix
    (.json, .md, .pdf)."""
    meters: Dict[str, TenantMeter] = {}
    for job in ledger.list_jobs(100000, org_id=org_id):
        run = ledger.get_latest_run(job["job_id"])
        if not run or not Path(run["metrics_path"]).exists():
            continue
        try:
            m = json.loads(Path(run["metrics_path"]).read_text(encoding="utf-8"))
        except ValueError:
            continue
        spec = json.loads(job["jobspec_json"])
        tenant = str(spec.get("tenant_id") or job["org_id"])
        meters.setdefault(tenant, TenantMeter(tenant)).accumulate(m)
    rep = {"generated_at": utc_now(), "gpu_hourly_cost": gpu_hourly_cost,
           "tenants": [mt.summary(gpu_hourly_cost) for mt in meters.values()],
           "targets": target_report(ledger, targets or [0.2, 0.3, 0.5], org_id)}
    out = Path(out_path)
    lines = [f"Savings report {rep['generated_at']} (GPU-hour ${gpu_hourly_cost:.2f})", ""]
    for t in rep["tenants"]:
        lines.append(f"{t['tenant_id']}: {t['total_requests']} requests, hit rate {t['amf_hit_rate']:.1%}, "
                     f"saved {t['total_saved_ms']:.0f} ms ({t['savings_pct']:.1f}%), ${t['cost_saved_usd']:.4f}")
    lines.append("")
    lines.append(f"achieved savings {rep['targets']['achieved_pct']:.1f}% over {rep['targets']['runs']} runs")
    for r in rep["targets"]["targets"]:
        lines.append(f"target {r['target_pct']:.0f}%: {'met' if r['met'] else 'not met'}, "
                     f"{r['additional_saved_ms_needed']:.0f} ms more needed")
    if out.suffix == ".pdf":
        write_pdf(out, lines)
    elif out.suffix == ".md":
        out.write_text("\n".join(["# " + lines[0]] + ["- " + l if l else "" for l in lines[1:]]) + "\n")
    else:
        out.write_text(json.dumps(rep, indent=2))
    return rep
