"""Control plane: accepts jobs, routes them to workers and answers the gateway's
status, KPI and billing queries.

``submit`` validates a jobspec (``prompt`` or ``messages``, ``max_tokens``,
``backend_id``, ``model``, ``deterministic``, ``policy``, optional
``idempotency_key``), canonicalises the prompt, derives

* ``prompt_hash`` -- sha256 of the canonical prompt;
* ``sampling_hash`` -- sha256 of the deterministic settings and ``max_tokens``;
* ``fingerprint_hash`` -- sha256 of the backend fingerprint and the pool key of the
  prompt's page-aligned prefix: two jobs with the same model and the same prefix share
  a KV snapshot;

checks the context budget, asks the :class:`~.router.ClusterRouter` for a worker and a
lane (a snapshot already recorded for the fingerprint upgrades the lane to a HIT),
inserts the job into the ledger and enqueues it. A repeated ``idempotency_key``
returns the existing job.

Reference: platform/runtime/cluster_router.py:108-316 (submit), :924-1298 (KPI,
billing and debug endpoints).
"""
from __future__ import annotations

import json
import os
import statistics
import uuid
from pathlib import Path
from typing import Any, Dict, List, Optional

from . import jobspec as jobspec_v1

from ..amf.keys import pool_key
from ..amf.prompt_policy import amf_prefix_tokens, amf_tenant
from .economics import TenantMeter, estimate_savings, target_report
from .ledger import canonical_json, sha256_hex
from .observability import GLOBAL_METRICS, utc_now
from .router import ClusterRouter, WorkerInfo, canonicalize


class JobError(ValueError):
    def __init__(self, msg: str, code: str = "BAD_REQUEST", status_code: int = 400):
        super().__init__(msg)
        self.code, self.status_code = code, status_code

    def to_payload(self) -> Dict[str, Any]:
        return {"error": str(self), "code": self.code}


def render_messages(messages: List[Dict[str, Any]]) -> str:
    return "".join(f"<|{m.get('role', 'user')}|>{m.get('content', '')}\n" for m in messages) + "<|assistant|>"


class ControlPlane:
    def __init__(self, ledger, workers: Dict[str, Any], *, node_id: str = "node-0", node_registry=None,
                 snapshot_index=None, coordinator=None, metrics=GLOBAL_METRICS, max_tokens_limit: int = 32768,
                 default_backend: str = "axr_engine", strict_jobspec: Optional[bool] = None):
        self.ledger = ledger
        self.workers = workers  # worker_id -> ClusterWorker (this node's)
        self.node_id = node_id
        self.nodes = node_registry
        self.index = snapshot_index
        self.coord = coordinator
        self.metrics = metrics
        self.max_tokens_limit = max_tokens_limit
        self.default_backend = default_backend
        # korith.jobspec.v1 only (KORITH_JOBSPEC_STRICT=1); otherwise v1 specs are checked
        # against the contract and the short form ({"prompt": ..., "max_tokens": ...}) is accepted
        self.strict_jobspec = (os.environ.get("KORITH_JOBSPEC_STRICT", "0") == "1" if strict_jobspec is None
                               else bool(strict_jobspec))
        infos = []
        for wid, w in workers.items():
            eng = getattr(getattr(w, "adapters", None), "engine", None)
            max_ctx = eng.cfg.max_model_len if eng is not None else 32768
            infos.append(WorkerInfo(wid, w.node_id, max_ctx=max_ctx, spec=getattr(eng, "spec", None) is not None))
        self.router = ClusterRouter(infos, coordinator=coordinator)

    # ------------------------------------------------------------------ jobs
    def _validate(self, job: Dict[str, Any]) -> Dict[str, Any]:
        if not isinstance(job, dict):
            raise JobError("jobspec must be a JSON object", "INVALID_JOBSPEC")
        if "schema_version" in job or self.strict_jobspec:
            errs = jobspec_v1.validate(job)
            if errs:
                raise JobError("invalid korith.jobspec.v1: " + "; ".join(errs), "INVALID_JOBSPEC")
            job = jobspec_v1.to_job(job)
        if "messages" in job and "prompt" not in job:
            if not isinstance(job["messages"], list):
                raise JobError("messages must be a list", "INVALID_JOBSPEC")
            job["prompt"] = render_messages(job["messages"])
        if not isinstance(job.get("prompt"), str) or not job["prompt"]:
            raise JobError("prompt (non-empty string) or messages required", "INVALID_JOBSPEC")
        mt = job.get("max_tokens", 64)
        if not isinstance(mt, int) or mt < 1 or mt > self.max_tokens_limit:
            raise JobError(f"max_tokens must be an integer in [1, {self.max_tokens_limit}]", "INVALID_JOBSPEC")
        for k in ("model", "deterministic", "policy"):
            if k in job and not isinstance(job[k], dict):
                raise JobError(f"{k} must be an object", "INVALID_JOBSPEC")
        job.setdefault("backend_id", self.default_backend)
        job.setdefault("deterministic", {"temperature": 0.0, "seed": 0})
        job.setdefault("policy", {})
        return job

    def fingerprint_of(self, job: Dict[str, Any], tokens: List[int]) -> Dict[str, Any]:
        worker = next(iter(self.workers.values()), None)
        fp: Dict[str, Any] = {"backend_id": job["backend_id"], "model": job.get("model", {})}
        if worker is not None:
            try:
                fp = dict(worker.adapters.get_adapter(job).get_fingerprint())
            except Exception:
                pass
        pre = tokens[: self.prefix_len(job, tokens)]
        fp["prefix_key"] = pool_key(pre) if pre else ""
        return fp

    @staticmethod
    def prefix_len(job: Dict[str, Any], tokens: List[int]) -> int:
        """Tokens of the prompt's reusable prefix (page-aligned, at least one token left
        to prefill): the job's ``amf_prefix_len`` if given, else the whole prompt up to
        ``KORITH_FINGERPRINT_PREFIX_TOKENS`` (default 32768)."""
        import os

        cap = int(job.get("amf_prefix_len") or os.environ.get("KORITH_FINGERPRINT_PREFIX_TOKENS", "32768"))
        return min(cap, len(tokens) - 1) // 16 * 16

    def submit(self, job: Dict[str, Any], org_id: str = "default", request_id: str = "",
               tenant_id: str = "default") -> str:
        job = self._validate(dict(job))
        if org_id == "default" and job.get("org_id"):  # korith.jobspec.v1 owner.org_id
            org_id = str(job["org_id"])
        job.setdefault("tenant_id", tenant_id)
        idem = job.get("idempotency_key")
        if idem:
            prev = self.ledger.find_job_by_idempotency(str(idem), org_id)
            if prev:
                return prev
        text = canonicalize(job["prompt"])
        toks = list(text.encode("utf-8"))
        if job.get("amf_prefix_len") is None:  # KORITH_AMF_PREFIX_EXTRACTION: key on the part before the last turn
            n = amf_prefix_tokens(toks, lambda s: list(s.encode("utf-8")))
            if n:
                job["amf_prefix_len"] = n
        fp = self.fingerprint_of(job, toks)
        fp["tenant_ns"] = amf_tenant(tenant_id, text)  # isolated, shared (patterns) or one namespace
        fp_hash = sha256_hex(canonical_json(fp))
        det = job["deterministic"]
        sampling_hash = sha256_hex(canonical_json({"det": det, "max_tokens": job.get("max_tokens", 64)}))
        job_id = uuid.uuid4().hex
        for wid, info in self.router.workers.items():  # load = queued + running jobs, in prompt tokens
            w = self.workers[wid]
            info.load = float(getattr(w, "queued_tokens", 0))
        route = self.router.submit(text, tenant_id, int(job.get("max_tokens", 64)), job=None, tokens=toks)
        lane = route.lane
        if self.index is not None and self.index.get_locations(fp_hash, org_id) and not lane.endswith("HIT"):
            lane = lane.replace("MISS", "HIT")
        if job.get("policy", {}).get("allow_spec") and not lane.startswith("SPEC"):
            lane = "SPEC_" + lane
        self.ledger.insert_job(job_id, utc_now(), job, fp, sha256_hex(text), fp_hash, idem, "queued", org_id)
        item = dict(job, job_id=job_id, org_id=org_id, tenant_id=tenant_id, prompt=text, prompt_tokens=len(toks),
                    lane=lane, fingerprint_hash=fp_hash, prompt_hash=sha256_hex(text), sampling_hash=sampling_hash,
                    request_id=request_id, n_ctx=route.worker.max_ctx, amf_prefix_len=self.prefix_len(job, toks),
                    routing={"kind": route.kind, "worker_id": route.worker.worker_id, "lane": lane,
                             "reasons": route.reasons, "source_node": route.source_node})
        self.workers[route.worker.worker_id].enqueue(item)
        self.metrics.inc("korith_jobs_submitted_total", 1, {"lane": lane, "org_id": org_id})
        return job_id

    def list_jobs(self, limit: int = 20, org_id: Optional[str] = None) -> List[Dict[str, Any]]:
        return [{"job_id": j["job_id"], "created_at": j["created_at"], "status": j["status"],
                 "fingerprint_hash": j["fingerprint_hash"]} for j in self.ledger.list_jobs(limit, org_id=org_id)]

    def get_job(self, job_id: str, org_id: Optional[str] = None) -> Optional[Dict[str, Any]]:
        j = self.ledger.get_job(job_id)
        if j is None or (org_id is not None and j["org_id"] != org_id):
            return None
        out = {k: j[k] for k in ("job_id", "created_at", "org_id", "status", "fingerprint_hash", "prompt_hash")}
        out["jobspec"] = json.loads(j["jobspec_json"])
        out["immutable"] = self.ledger.verify_job(job_id)
        run = self.ledger.get_latest_run(job_id)
        if run:
            out.update({k: run[k] for k in ("metrics_path", "events_path", "output_path", "log_path", "exit_code",
                                            "started_at", "finished_at")})
            p = Path(run["output_path"])
            out["output_text"] = p.read_text(encoding="utf-8") if p.exists() else ""
        return out

    def restore(self, job_id: str, org_id: Optional[str] = None, request_id: str = "") -> Dict[str, Any]:
        """Re-run a finished job as a HIT on its snapshot (the KV is replayed, not prefilled)."""
        j = self.ledger.get_job(job_id)
        if j is None or (org_id is not None and j["org_id"] != org_id):
            return {"restored": False, "error": "job not found"}
        snap = self.ledger.get_snapshot_for_job(job_id)
        if snap is None:
            return {"restored": False, "error": "job has no snapshot"}
        spec = json.loads(j["jobspec_json"])
        spec.pop("idempotency_key", None)
        new_id = self.submit(spec, j["org_id"], request_id, spec.get("tenant_id", j["org_id"]))
        return {"restored": True, "job_id": new_id, "snapshot_id": snap["snapshot_id"],
                "fingerprint_hash": j["fingerprint_hash"]}

    # ------------------------------------------------------------------ status
    def get_workers(self) -> List[Dict[str, Any]]:
        return [w.health() for w in self.workers.values()]

    def queue_status(self) -> List[Dict[str, Any]]:
        return [w.queue_status() for w in self.workers.values()]

    def capabilities(self) -> Dict[str, Any]:
        out = {}
        for wid, w in self.workers.items():
            try:
                a = w.adapters.get_adapter({"backend_id": self.default_backend})
                out[wid] = {"backend_id": a.backend_id, **a.get_capabilities().as_dict()}
            except Exception as e:
                out[wid] = {"error": str(e)}
        return out

    def cluster_nodes(self) -> List[Dict[str, Any]]:
        return self.nodes.list_nodes() if self.nodes is not None else [{"node_id": self.node_id}]

    def snapshot_locations(self, fingerprint_hash: str, org_id: str) -> Dict[str, Any]:
        locs = self.index.get_locations(fingerprint_hash, org_id) if self.index is not None else \
            self.ledger.list_snapshot_locations(fingerprint_hash, org_id)
        return {"fingerprint_hash": fingerprint_hash, "locations": locs}

    def routing_debug(self, fingerprint_hash: str, org_id: str) -> Dict[str, Any]:
        locs = self.snapshot_locations(fingerprint_hash, org_id)["locations"]
        local = [l for l in locs if l["node_id"] == self.node_id]
        return {"fingerprint_hash": fingerprint_hash, "snapshot_local": bool(local), "locations": locs,
                "router_stats": dict(self.router.stat),
                "workers": [{"worker_id": w.worker_id, "load": w.load} for w in self.router.workers.values()]}

    def replay_status(self, fingerprint_hash: str) -> Dict[str, Any]:
        w = next(iter(self.workers.values()), None)
        if w is None:
            return {"fingerprint_hash": fingerprint_hash, "replay_allowed": True}
        return w.replay.status(fingerprint_hash)

    def spec_status(self, fingerprint_hash: str, org_id: Optional[str] = None) -> Dict[str, Any]:
        g = self.ledger.get_spec_governance(fingerprint_hash) or {}
        w = next(iter(self.workers.values()), None)
        return {"fingerprint_hash": fingerprint_hash, "governance": g,
                "spec_allowed": w.spec_gov.allowed(fingerprint_hash) if w else True,
                "controller": w.spec_k.metrics() if w else {}}

    def kernels_status(self) -> Dict[str, Any]:
        """Which native modules this process loaded, and whether CUDA is usable."""
        import sys

        mods = {}
        for name in ("axropus_deploy_b200._C", "axropus_deploy_b200._native"):
            m = sys.modules.get(name)
            mods[name] = {"loaded": m is not None, "file": getattr(m, "__file__", None)}
        try:
            import torch

            cuda = torch.cuda.is_available()
            dev = torch.cuda.get_device_name(0) if cuda else None
        except Exception:
            cuda, dev = False, None
        return {"cuda": cuda, "device": dev, "modules": mods, "arch": "sm_100a"}

    def _run_metrics(self, org_id: Optional[str], limit: int, tenant_id: Optional[str] = None):
        for j in self.ledger.list_jobs(limit, org_id=org_id):
            if tenant_id and json.loads(j["jobspec_json"]).get("tenant_id", j["org_id"]) != tenant_id:
                continue
            run = self.ledger.get_latest_run(j["job_id"])
            if not run or not Path(run["metrics_path"]).exists():
                continue
            try:
                yield j, json.loads(Path(run["metrics_path"]).read_text(encoding="utf-8"))
            except ValueError:
                continue

    def kpi_summary(self, org_id: Optional[str] = None, limit: int = 500, gpu_hourly_cost: float = 2.5) -> Dict:
        ttft_hit, ttft_miss, saved, total = [], [], 0.0, 0.0
        hits = n = 0
        for _, m in self._run_metrics(org_id, limit):
            n += 1
            perf, amf = m.get("perf") or {}, m.get("amf") or {}
            (ttft_hit if amf.get("decision") == "hit" else ttft_miss).append(float(perf.get("ttft_ms", 0.0)))
            hits += amf.get("decision") == "hit"
            s = estimate_savings(m, gpu_hourly_cost)
            saved += s["saved_ms"]
            total += s["total_ms"]

        def q(xs, p):
            if not xs:
                return None
            xs = sorted(xs)
            return xs[min(len(xs) - 1, int(round(p / 100 * (len(xs) - 1))))]

        per_ms = gpu_hourly_cost / 3_600_000.0
        return {"runs": n, "hit_rate": hits / n if n else 0.0,
                "ttft_hit_ms": {"p50": q(ttft_hit, 50), "p99": q(ttft_hit, 99)},
                "ttft_miss_ms": {"p50": q(ttft_miss, 50), "p99": q(ttft_miss, 99)},
                "speedup_p50": (q(ttft_miss, 50) / q(ttft_hit, 50)) if ttft_hit and ttft_miss and q(ttft_hit, 50)
                else None,
                "saved_ms": saved, "served_ms": total, "cost_saved_usd": saved * per_ms,
                "cost_served_usd": total * per_ms,
                "mean_ttft_ms": statistics.fmean(ttft_hit + ttft_miss) if (ttft_hit or ttft_miss) else None}

    def tenant_metrics(self, tenant_id: str, org_id: Optional[str] = None, gpu_hourly_cost: float = 2.5) -> Dict:
        meter = TenantMeter(tenant_id)
        for _, m in self._run_metrics(org_id, 100000, tenant_id):
            meter.accumulate(m)
        return meter.summary(gpu_hourly_cost)

    def billing_report(self, org_id: Optional[str] = None, tenant_id: str = "", limit: int = 5000,
                       gpu_hourly_cost: float = 2.5) -> Dict[str, Any]:
        meters: Dict[str, TenantMeter] = {}
        for j, m in self._run_metrics(org_id, limit, tenant_id or None):
            t = json.loads(j["jobspec_json"]).get("tenant_id", j["org_id"])
            meters.setdefault(t, TenantMeter(t)).accumulate(m)
        return {"org_id": org_id, "generated_at": utc_now(), "gpu_hourly_cost": gpu_hourly_cost,
                "tenants": [mt.summary(gpu_hourly_cost) for mt in meters.values()],
                "targets": target_report(self.ledger, [0.2, 0.3, 0.5], org_id, limit)}
