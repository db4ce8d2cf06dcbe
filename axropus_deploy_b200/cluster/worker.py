"""Cluster worker: one per GPU engine. Takes jobs from four lane queues, runs them on a
backend adapter and records everything the control plane reports on.

Lanes and scheduling. Jobs arrive tagged ``SPEC_HIT``, ``HIT``, ``SPEC_MISS`` or
``MISS`` (the router's prediction). The worker serves the lanes by weighted round
robin: in each round a lane may start up to its budget of jobs
(``KORITH_SPEC_PRIORITY`` 4, ``KORITH_HIT_PRIORITY`` 3, half the spec budget for
``SPEC_MISS``, ``KORITH_MISS_PRIORITY`` 1); empty lanes give their turn away, and a new
round starts when every non-empty lane has spent its budget. Restores are short and
free GPU time for everybody, so hits go first without starving misses.

A job (``_process``):

1. answers from the decode cache when the same deterministic job already ran;
2. finds the KV snapshot of its fingerprint when replay is allowed for it: a local
   one is validated (metadata sidecar, checksum) and replayed; a snapshot on another
   node is fetched over HTTP and stored in the fastest snapshot tier when moving it
   beats recomputing the prefix (``estimate_transfer_ms`` vs the measured cold-prefill
   cost), else the job runs as a miss;
3. runs ``run_speculative`` (SPEC lanes, speculation allowed, depth from the
   :class:`~.runtime.SpecKController`), ``run_accel`` or ``run_baseline`` (forced
   miss, accelerations off);
4. writes ``output.txt``, ``metrics.json`` (perf, amf, spec, savings, routing),
   ``events.jsonl`` and ``run.log``; inserts the run, the new snapshot (with its
   sidecar) and its location into the ledger; registers the prefix with the AMF
   coordinator; updates the replay / speculation governance and the metrics registry.

Failures mark the job ``failed`` with the error in the run log; the worker keeps going.
With ``concurrency`` > 1 several threads take jobs at once; over an adapter whose engine is
driven by an ``EngineService`` their requests share engine steps (continuous batching).

Reference: platform/runtime/cluster_worker.py:455-621 (lane budgets), :924-1114 and
:2170-2410 (snapshot transfer into the tiered cache), :1413-1475 (run selection),
:816-868 and :2412-3361 (governance, metrics, coordinator heartbeat).
"""
from __future__ import annotations

import hashlib
import os
import threading
import traceback
import uuid
from pathlib import Path
from typing import Any, Dict, List, Optional

from .adapters import AdapterRegistry
from .engine_client import validate_snapshot_metadata, write_snapshot_metadata
from .nodes import estimate_transfer_ms, fetch_snapshot_bytes, should_transfer_snapshot, store_snapshot_bytes
from .observability import GLOBAL_METRICS, ArtifactStore, emit_log, error_fields, utc_now
from .queues import InProcQueue
from .runtime import DecodeCache, ReplayGovernor, SpecGovernor, SpecKController

LANES = ("SPEC_HIT", "HIT", "SPEC_MISS", "MISS")


def _env_int(name: str, default: int) -> int:
    try:
        return max(1, int(os.environ.get(name, "") or default))
    except ValueError:
        return default


def lane_budgets() -> Dict[str, int]:
    spec = _env_int("KORITH_SPEC_PRIORITY", 4)
    return {"SPEC_HIT": spec, "HIT": _env_int("KORITH_HIT_PRIORITY", 3), "SPEC_MISS": max(1, spec // 2),
            "MISS": _env_int("KORITH_MISS_PRIORITY", 1)}


class ClusterWorker:
    def __init__(self, worker_id: str, node_id: str, adapters: AdapterRegistry, ledger, artifacts: ArtifactStore, *,
                 snapshot_index=None, node_registry=None, coordinator=None, decode_cache: Optional[DecodeCache] = None,
                 metrics=GLOBAL_METRICS, snapshot_dir: Optional[str] = None, link_gbps: Optional[float] = None,
                 rtt_ms: Optional[float] = None, transfer_threshold: Optional[float] = None, gpu_index: int = 0,
                 queue_factory=None, concurrency: int = 1, policy=None, uploader=None):
        self.worker_id, self.node_id, self.gpu_index = worker_id, node_id, gpu_index
        self.concurrency = max(1, int(concurrency))  # jobs in flight (batched by an EngineService)
        self.policy = policy  # optional decision layer (PolicyOrchestrator): fail-closed hooks around each run
        self.uploader = uploader  # optional object store (S3 / MinIO) that receives each finished job's files
        self.adapters = adapters
        self.ledger = ledger
        self.artifacts = artifacts
        self.index = snapshot_index
        self.nodes = node_registry
        self.coord = coordinator
        self.dcache = decode_cache
        self.metrics = metrics
        self.snapshot_dir = Path(snapshot_dir or os.environ.get("KORITH_SNAPSHOT_RAM_DIR", "")
                                 or artifacts.base / "_snapshots")
        mbps = float(os.environ.get("KORITH_SNAPSHOT_BW_MBPS", "0") or 0)
        self.link_gbps = link_gbps if link_gbps is not None else (mbps / 1e3 if mbps > 0 else 12.5)
        self.rtt_ms = rtt_ms if rtt_ms is not None else float(os.environ.get("KORITH_SNAPSHOT_RTT_MS", "1") or 1)
        self.threshold = transfer_threshold if transfer_threshold is not None else \
            float(os.environ.get("KORITH_TRANSFER_VS_RECOMPUTE_THRESHOLD", "0.8") or 0.8)
        self.accel_enabled = os.environ.get("KORITH_ACCEL_ENABLED", "1").lower() not in ("0", "false", "no")
        self.replay = ReplayGovernor(ledger)
        self.spec_gov = SpecGovernor(ledger)
        self.spec_k = SpecKController(_env_int("KORITH_SPEC_K", SpecKController.DEFAULT_K))
        # one queue per lane: in-process by default; with a factory (e.g. one SqliteQueue per
        # lane) jobs survive the worker -- a job taken but never acked (the worker died in
        # the middle of it) becomes ready again after the queue's visibility timeout
        self.queues: Dict[str, Any] = {l: (queue_factory(l) if queue_factory else InProcQueue()) for l in LANES}
        self.budget = lane_budgets()
        self._left = dict(self.budget)
        self._mu = threading.Lock()
        self._cv = threading.Condition(self._mu)
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.inflight = 0
        self.queued_tokens = 0  # prompt + output tokens of queued and running jobs (router load)
        self.done = 0
        self.failed = 0
        self.cold_ms_per_token = 0.0  # prices a recompute in the transfer decision

    # ------------------------------------------------------------------ queues
    def enqueue(self, job: Dict[str, Any]) -> None:
        lane = str(job.get("lane", "MISS")).upper()
        with self._cv:
            self.queues[lane if lane in self.queues else "MISS"].enqueue(job)
            self.queued_tokens += int(job.get("prompt_tokens", 0)) + int(job.get("max_tokens", 0))
            self._cv.notify()
        self.metrics.set_gauge("korith_worker_queue_depth", self.depth(lane), {"worker": self.worker_id,
                                                                               "lane": lane})

    @staticmethod
    def _ready(q) -> int:
        st = q.stats()
        return int(st.get("ready", 0)) + int(st.get("delayed", 0))

    def depth(self, lane: Optional[str] = None) -> int:
        if lane is not None:
            q = self.queues.get(lane)
            return self._ready(q) if q is not None else 0
        return sum(self._ready(q) for q in self.queues.values())

    def queue_status(self) -> Dict[str, Any]:
        return {"worker_id": self.worker_id, "depths": {l: self._ready(q) for l, q in self.queues.items()},
                "budget_left": dict(self._left), "inflight": self.inflight, "done": self.done, "failed": self.failed}

    def _next(self) -> Optional[tuple]:
        """(lane, item id, job) by weighted round robin over the lanes that have work
        (caller holds the lock)."""
        for _ in range(2):
            for lane in LANES:
                if self._left[lane] > 0:
                    got = self.queues[lane].dequeue()
                    if got is not None:
                        self._left[lane] -= 1
                        return lane, got[0], got[1]
            if self.depth() == 0:
                return None
            self._left = dict(self.budget)  # every lane with work spent its budget: new round
        return None

    # ------------------------------------------------------------------ loop
    def run_once(self, block: bool = False, timeout: float = 0.5) -> Optional[Dict[str, Any]]:
        with self._cv:
            got = self._next()
            if got is None and block:
                self._cv.wait(timeout)
                got = self._next()
            if got is None:
                return None
            self.inflight += 1
        lane, iid, job = got
        try:
            out = self._process(job)
            self.queues[lane].ack(iid)  # terminal state (succeeded or failed) recorded in the ledger
            return out
        finally:
            with self._mu:
                self.inflight -= 1
                self.queued_tokens = max(0, self.queued_tokens - int(job.get("prompt_tokens", 0))
                                         - int(job.get("max_tokens", 0)))

    def drain(self) -> List[Dict[str, Any]]:
        out = []
        while True:
            r = self.run_once()
            if r is None:
                return out
            out.append(r)

    def start(self) -> "ClusterWorker":
        def loop():
            while not self._stop.is_set():
                self.run_once(block=True)

        self._threads = [threading.Thread(target=loop, name=f"worker-{self.worker_id}-{i}", daemon=True)
                         for i in range(self.concurrency)]
        for t in self._threads:
            t.start()
        self._thread = self._threads[0]
        return self

    def stop(self) -> None:
        self._stop.set()
        with self._cv:
            self._cv.notify_all()
        for t in getattr(self, "_threads", []):
            t.join(timeout=10)

    def health(self) -> Dict[str, Any]:
        return {"worker_id": self.worker_id, "node_id": self.node_id, "gpu_index": self.gpu_index,
                "status": "busy" if self.inflight else "idle", "queue_depth": self.depth(), "done": self.done,
                "failed": self.failed, "spec": self.spec_k.metrics()}

    # ------------------------------------------------------------------ snapshots
    def _local_snapshot(self, fp: str, org: str, fingerprint: Dict[str, str], n_ctx: int) -> Optional[str]:
        if self.index is None:
            return None
        for loc in self.index.get_locations(fp, org):
            if loc["node_id"] != self.node_id:
                continue
            ok, reason, _ = validate_snapshot_metadata(loc["snapshot_path"], fingerprint_hash=fp,
                                                       model_hash=fingerprint.get("model_hash", ""),
                                                       tokenizer_hash=fingerprint.get("tokenizer", ""),
                                                       kv_layout_version=fingerprint.get("kv_layout", ""),
                                                       n_ctx=n_ctx)
            if ok:
                self.index.mark_used(fp, org, self.node_id, loc["snapshot_id"])
                return loc["snapshot_path"]
            if reason == "snapshot_checksum_mismatch":
                self.replay.record(fp, 0.0, corrupted=True)
        return None

    def _remote_snapshot(self, job: Dict[str, Any], fp: str, org: str, fingerprint: Dict[str, str],
                         n_ctx: int, events: list) -> Optional[str]:
        if self.index is None or self.nodes is None:
            return None
        remote = [l for l in self.index.get_locations(fp, org) if l["node_id"] != self.node_id]
        if not remote:
            return None
        baseline_ms = job.get("prompt_tokens", 0) * self.cold_ms_per_token
        best = None
        for loc in remote:
            node = self.nodes.get_node(loc["node_id"])
            if node is None:
                continue
            ms = estimate_transfer_ms(int(loc["size_bytes"]), self.link_gbps, self.rtt_ms, loc["storage_tier"])
            if best is None or ms < best[0]:
                best = (ms, loc, node)
        if best is None:
            return None
        ms, loc, node = best
        go = should_transfer_snapshot(job.get("lane", ""), True, ms, baseline_ms, self.threshold)
        events.append({"event": "transfer_decision", "transfer_ms": ms, "recompute_ms": baseline_ms,
                       "source_node": loc["node_id"], "transfer": go})
        if not go:
            return None
        try:
            data, meta = fetch_snapshot_bytes(node["host"], node["router_port"], fp, org)
        except Exception as e:  # the source node went away: run as a miss
            events.append({"event": "transfer_failed", **error_fields(e)})
            return None
        path = self.snapshot_dir / org / f"{fp}.amfk"
        tok = bytes.fromhex(meta.get("tokens_hex", "")) if meta.get("tokens_hex") else None
        store_snapshot_bytes(path, data, tok)
        write_snapshot_metadata(path, fingerprint_hash=fp, model_hash=fingerprint.get("model_hash", ""),
                                tokenizer_hash=fingerprint.get("tokenizer", ""), backend_id=fingerprint["backend_id"],
                                n_ctx=n_ctx, kv_layout_version=fingerprint.get("kv_layout", ""), created_at=utc_now())
        sid = meta.get("snapshot_id") or uuid.uuid4().hex
        self.index.upsert_location(fp, sid, org, self.node_id, self.worker_id, str(path), len(data))
        events.append({"event": "snapshot_transferred", "bytes": len(data), "from": loc["node_id"]})
        self.metrics.inc("korith_snapshot_transfers_total", 1, {"worker": self.worker_id})
        return str(path)

    # ------------------------------------------------------------------ one job
    def _process(self, job: Dict[str, Any]) -> Dict[str, Any]:
        job_id, org = job["job_id"], job.get("org_id", "default")
        fp = job.get("fingerprint_hash", "")
        lane = str(job.get("lane", "MISS")).upper()
        paths = self.artifacts.init_job(job_id, org)
        events: List[Dict[str, Any]] = [{"event": "dequeued", "lane": lane, "worker": self.worker_id, "ts": utc_now()}]
        started = utc_now()
        self.ledger.update_status(job_id, "running")
        det = job.get("deterministic") or {}
        policy = job.get("policy") or {}
        n_ctx = int(job.get("n_ctx", 0) or 0)
        result: Dict[str, Any] = {}
        exit_code = 0
        try:
            adapter = self.adapters.get_adapter(job)
            fingerprint = adapter.get_fingerprint()
            caps = adapter.get_capabilities().as_dict()
            cache_key = dict(org_id=org, backend_id=adapter.backend_id, fingerprint_hash=fp,
                             prompt_hash=job.get("prompt_hash", ""), sampling_hash=job.get("sampling_hash", ""))
            cached = self.dcache.get(**cache_key) if (self.dcache is not None and
                                                       float(det.get("temperature", 0.0)) == 0.0) else None
            if cached is not None:
                events.append({"event": "decode_cache_hit"})
                result = {"output_text": cached["output_text"], "tokens_out": cached["tokens_out"],
                          "perf": {"total_ms": 0.0, "ttft_ms": 0.0, "prefill_ms": 0.0, "decode_ms": 0.0},
                          "amf": {"decision": "hit", "tier": "decode_cache", "saved_ms": cached["total_ms"]},
                          "spec": {}}
            else:
                snap_in = None
                replay = self.replay.status(fp)
                force_miss = bool(policy.get("force_miss", False))
                if caps.get("KV_REPLAY") and replay["replay_allowed"] and not force_miss and lane.endswith("HIT"):
                    snap_in = self._local_snapshot(fp, org, fingerprint, n_ctx) or \
                        self._remote_snapshot(job, fp, org, fingerprint, n_ctx, events)
                events.append({"event": "snapshot", "path": snap_in, "replay_allowed": replay["replay_allowed"]})
                ptok = self.policy.before_job(job) if self.policy is not None else None
                spec_gate = self.spec_k.gate(caps, policy) if lane.startswith("SPEC") else {"enabled": False}
                if spec_gate["enabled"] and not self.spec_gov.allowed(fp):
                    spec_gate = {"enabled": False, "reason": "governance"}
                art = {"snapshot": str(paths["snapshot"])} if caps.get("KV_REPLAY") else {}
                args = (job["prompt"], int(job.get("max_tokens", 64)), det, policy, art, snap_in)
                ecfg = {"amf_prefix_len": job.get("amf_prefix_len")}
                if force_miss or not self.accel_enabled:
                    mode, result = "baseline", adapter.run_baseline(*args)
                elif spec_gate["enabled"]:
                    mode, result = "speculative", adapter.run_speculative(*args, spec_cfg={"k": spec_gate["k"]},
                                                                          engine_cfg=ecfg)
                else:
                    mode, result = "accel", adapter.run_accel(*args, engine_cfg=ecfg)
                events.append({"event": "run", "mode": mode})
                amf = result.get("amf") or {}
                if amf.get("tier") == "cold" and job.get("prompt_tokens"):
                    rate = result["perf"]["prefill_ms"] / max(1, job["prompt_tokens"])
                    self.cold_ms_per_token = rate if not self.cold_ms_per_token else \
                        0.8 * self.cold_ms_per_token + 0.2 * rate
                if snap_in or amf.get("decision") == "hit":
                    self.replay.record(fp, float(amf.get("saved_ms", 0.0)))
                sp = result.get("spec") or {}
                if mode == "speculative" and sp:
                    drafted, accepted = int(sp.get("drafted", 0)), int(sp.get("accepted", 0))
                    self.spec_k.update(drafted, accepted, 0.0, float(result["perf"].get("tok_s", 0.0)))
                    self.spec_gov.record(fp, org, accepted / max(1, drafted))
                if self.policy is not None:
                    self.policy.after_job(ptok, result, mode)
                if self.dcache is not None and float(det.get("temperature", 0.0)) == 0.0:
                    self.dcache.put(**cache_key, output_text=result.get("output_text", ""),
                                    tokens_out=int(result.get("tokens_out", 0)),
                                    decode_ms=float(result["perf"].get("decode_ms", 0.0)),
                                    total_ms=float(result["perf"].get("total_ms", 0.0)))
                self._record_snapshot(job, result, paths, fingerprint, n_ctx, events)
        except Exception as e:
            exit_code = 1
            events.append({"event": "failed", **error_fields(e)})
            Path(paths["log"]).write_text(traceback.format_exc(), encoding="utf-8")
        finished = utc_now()
        metrics = {"job_id": job_id, "worker_id": self.worker_id, "node_id": self.node_id, "lane": lane,
                   "perf": result.get("perf", {}), "amf": result.get("amf", {}), "spec": result.get("spec", {}),
                   "tokens_out": result.get("tokens_out", 0), "routing": job.get("routing", {}),
                   "savings": {"prefill_saved_ms": float((result.get("amf") or {}).get("saved_ms", 0.0)),
                               "spec_saved_ms": float((result.get("spec") or {}).get("saved_ms", 0.0)),
                               "kernels_saved_ms": 0.0}}
        self.artifacts.write_json(paths["metrics"], metrics)
        Path(paths["output"]).write_text(result.get("output_text", ""), encoding="utf-8")
        for ev in events:
            self.artifacts.append_event(paths["events"], ev)
        if exit_code == 0:
            emit_log("worker", "job_done", {"job_id": job_id, "lane": lane}, artifact_log=Path(paths["log"]),
                     echo=False)
        if self.uploader is not None:
            try:  # the local files stay authoritative; a failed upload is counted, not fatal
                self.uploader.upload_job(job_id, org)
                self.metrics.inc("korith_artifact_uploads_total", 1, {"status": "ok"})
            except Exception as e:
                self.metrics.inc("korith_artifact_uploads_total", 1, {"status": "failed"})
                emit_log("worker", "artifact_upload_failed", {"job_id": job_id, **error_fields(e)}, echo=False)
        self.ledger.insert_run(uuid.uuid4().hex, job_id, started, finished, exit_code, str(paths["metrics"]),
                               str(paths["events"]), str(paths["output"]), str(paths["log"]), org_id=org)
        self.ledger.update_status(job_id, "succeeded" if exit_code == 0 else "failed")
        with self._mu:
            self.done += exit_code == 0
            self.failed += exit_code != 0
        self.metrics.inc("korith_jobs_total", 1, {"lane": lane, "status": "ok" if exit_code == 0 else "failed",
                                                  "org_id": org})
        self.metrics.inc("korith_amf_saved_ms_total", float((result.get("amf") or {}).get("saved_ms", 0.0)))
        return {"job_id": job_id, "exit_code": exit_code, **metrics, "output_text": result.get("output_text", "")}

    def _record_snapshot(self, job, result, paths, fingerprint, n_ctx, events) -> None:
        snap = result.get("snapshot_path")
        if not snap or not Path(snap).exists():
            return
        fp, org = job.get("fingerprint_hash", ""), job.get("org_id", "default")
        write_snapshot_metadata(snap, fingerprint_hash=fp, model_hash=fingerprint.get("model_hash", ""),
                                tokenizer_hash=fingerprint.get("tokenizer", ""), backend_id=fingerprint["backend_id"],
                                n_ctx=n_ctx, kv_layout_version=fingerprint.get("kv_layout", ""), created_at=utc_now())
        sid = hashlib.sha256(f"{fp}:{self.node_id}".encode()).hexdigest()[:24]
        self.ledger.insert_snapshot(sid, job["job_id"], fp, snap, utc_now(), org_id=org)
        if self.index is not None:
            self.index.upsert_location(fp, sid, org, self.node_id, self.worker_id, snap, Path(snap).stat().st_size)
        if self.coord is not None:
            try:
                if hasattr(self.coord, "base"):
                    self.coord.register(fp, self.node_id, self.worker_id, tenant_id=org)
                else:
                    self.coord.register(org, fp, self.node_id, self.worker_id)
            except Exception:  # coordinator outage: locality only
                pass
        events.append({"event": "snapshot_saved", "path": snap, "tokens": result.get("snapshot_tokens", 0)})
