"""Platform command line (``python -m axropus_deploy_b200.cluster``).

* ``node``         -- one node of the cluster: an engine + worker per visible GPU (or one
                      CPU worker), the control plane, the HTTP gateway and the node's
                      snapshot server, registered in the node registry;
* ``coordinator``  -- the AMF coordinator service;
* ``create-key``   -- issue an API key (printed once) into the ledger;
* ``report``       -- savings report over the ledger (.json / .md / .pdf);
* ``apply-config`` -- print the ``KORITH_*`` variables a platform YAML/JSON file sets.

Reference: platform/korith_platform.py:46-525 (the platform CLI), platform/runtime/
worker_service.py / router_service.py (service mains).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time


def _build_node(a):
    import torch

    from ..config import AxropusConfig
    from ..server.app import build_engine
    from .adapters import AdapterRegistry
    from .control import ControlPlane
    from .coordinator import CoordinatorClient
    from .pgledger import build_ledger
    from .nodes import NodeRegistry, NodeServer, SnapshotIndex
    from .observability import ArtifactStore
    from .runtime import DecodeCache
    from ..server.service import EngineService
    from .netqueues import build_queue
    from .worker import ClusterWorker

    ledger = build_ledger(a.db)
    redis_url = os.environ.get("KORITH_REDIS_URL", "")
    index = SnapshotIndex(ledger, redis_url=os.environ.get("KORITH_SNAPSHOT_INDEX_REDIS_URL", redis_url))
    nodes = NodeRegistry(a.node_db, redis_url=os.environ.get("KORITH_NODE_REGISTRY_REDIS_URL", redis_url))
    coord = CoordinatorClient(a.coordinator) if a.coordinator else None
    art = ArtifactStore(a.artifacts)
    uploader = None
    if os.environ.get("KORITH_ARTIFACT_BACKEND", "local").strip().lower() in ("s3", "minio"):
        from .objstore import build_artifacts

        uploader = build_artifacts(a.artifacts)  # jobs' files are written locally, then copied to the bucket
    gpus = list(range(torch.cuda.device_count())) if torch.cuda.is_available() else [None]
    workers = {}
    for g in gpus[: a.max_workers]:
        if g is not None:
            torch.cuda.set_device(g)
        eng = build_engine(AxropusConfig.load(None, {"model": a.model, "device": f"cuda:{g}" if g is not None
                                                     else "cpu"}))
        wid = f"{a.node_id}-gpu{g if g is not None else 'cpu'}"
        svc = EngineService(eng)  # jobs of this GPU share engine steps (continuous batching)
        # KORITH_QUEUE_BACKEND (sqlite / redis / redis_streams / nats / sqs / inproc) picks the lane queues;
        # unset keeps them in this process
        qf = ((lambda lane, wid=wid: build_queue(f"{wid}:{lane}")) if os.environ.get("KORITH_QUEUE_BACKEND")
              else None)
        workers[wid] = ClusterWorker(wid, a.node_id, AdapterRegistry(eng, service=svc), ledger, art,
                                     snapshot_index=index, node_registry=nodes, coordinator=coord,
                                     decode_cache=DecodeCache(os.path.join(a.artifacts, "decode_cache.db")),
                                     gpu_index=g or 0, concurrency=a.jobs_per_worker, queue_factory=qf,
                                     uploader=uploader)
    plane = ControlPlane(ledger, workers, node_id=a.node_id, node_registry=nodes, snapshot_index=index,
                         coordinator=coord)
    status = lambda: {"gpu_count": len(gpus), "inflight": sum(w.inflight for w in workers.values()),  # noqa: E731
                      "queue_depth_hit": sum(w.depth("HIT") + w.depth("SPEC_HIT") for w in workers.values()),
                      "queue_depth_miss": sum(w.depth("MISS") + w.depth("SPEC_MISS") for w in workers.values())}
    server = NodeServer(a.node_id, index, a.host, a.node_port, registry=nodes, status=status)
    return plane, workers, server


def main(argv=None) -> int:
    if os.environ.get("KORITH_CONFIG"):
        from .runtime import apply_config_to_env, load_platform_config

        # the file fills KORITH_* variables that are not set yet; it is applied before the
        # argument defaults below read them
        apply_config_to_env(load_platform_config(os.environ["KORITH_CONFIG"]))
    p = argparse.ArgumentParser(prog="axropus-platform")
    sub = p.add_subparsers(dest="cmd", required=True)
    n = sub.add_parser("node")
    n.add_argument("--node-id", default=os.environ.get("KORITH_NODE_ID", "node-0"))
    n.add_argument("--host", default=os.environ.get("KORITH_NODE_HOST", "127.0.0.1"))
    n.add_argument("--port", type=int, default=8000)
    n.add_argument("--node-port", type=int, default=int(os.environ.get("KORITH_NODE_ROUTER_PORT", "8100")))
    n.add_argument("--model", default=os.environ.get("KORITH_DEFAULT_MODEL_ID", "tiny128"))
    n.add_argument("--db", default=os.environ.get("KORITH_PLATFORM_DB", "platform_data/ledger.db"))
    n.add_argument("--node-db", default=os.environ.get("KORITH_NODE_REGISTRY_DB", "platform_data/nodes.db"))
    n.add_argument("--artifacts", default=os.environ.get("KORITH_PLATFORM_ARTIFACTS", "platform_data/artifacts"))
    n.add_argument("--coordinator", default=os.environ.get("AMF_COORDINATOR_URL", ""))
    n.add_argument("--max-workers", type=int, default=8)
    n.add_argument("--jobs-per-worker", type=int, default=8, help="jobs in flight per GPU, batched by its engine")
    c = sub.add_parser("coordinator")
    c.add_argument("--db", default="platform_data/coordinator.db")
    c.add_argument("--host", default="127.0.0.1")
    c.add_argument("--port", type=int, default=8200)
    k = sub.add_parser("create-key")
    k.add_argument("--db", default=os.environ.get("KORITH_PLATFORM_DB", "platform_data/ledger.db"))
    k.add_argument("--key-id", required=True)
    k.add_argument("--org-id", required=True)
    k.add_argument("--rpm", type=int, default=600)
    k.add_argument("--tpm", type=int, default=120000)
    r = sub.add_parser("report")
    r.add_argument("--db", default=os.environ.get("KORITH_PLATFORM_DB", "platform_data/ledger.db"))
    r.add_argument("--out", required=True)
    r.add_argument("--gpu-hourly-cost", type=float, default=2.5)
    r.add_argument("--org-id", default=None)
    ac = sub.add_parser("apply-config")
    ac.add_argument("path")
    a = p.parse_args(argv)

    if a.cmd == "apply-config":
        from .runtime import apply_config_to_env, load_platform_config

        env: dict = {}
        print(json.dumps(apply_config_to_env(load_platform_config(a.path), env), indent=2))
        return 0
    for path in (getattr(a, "db", None), getattr(a, "node_db", None)):
        if path and os.path.dirname(path):
            os.makedirs(os.path.dirname(path), exist_ok=True)
    if a.cmd == "create-key":
        from .gateway import issue_api_key
        from .pgledger import build_ledger

        print(issue_api_key(build_ledger(a.db), a.key_id, a.org_id, a.rpm, a.tpm))
        return 0
    if a.cmd == "report":
        from .economics import write_report
        from .pgledger import build_ledger

        rep = write_report(build_ledger(a.db), a.out, a.gpu_hourly_cost, a.org_id)
        print(json.dumps(rep["targets"], indent=2))
        return 0
    if a.cmd == "coordinator":
        from .coordinator import AmfCoordinator, serve_coordinator

        httpd, port = serve_coordinator(AmfCoordinator(a.db), a.host, a.port)
        print(f"coordinator on {a.host}:{port}", flush=True)
        while True:
            time.sleep(3600)
    from .gateway import serve

    plane, workers, server = _build_node(a)
    server.start()
    for w in workers.values():
        w.start()
    print(f"node {a.node_id}: gateway {a.host}:{a.port}, snapshots {server.host}:{server.port}, "
          f"{len(workers)} worker(s)", flush=True)
    try:
        serve(plane, a.host, a.port, block=True)
    finally:
        for w in workers.values():
            w.stop()
        server.stop()
    return 0


if __name__ == "__main__":
    sys.exit(main())
