"""Control plane on CPU: coordinator index over HTTP (register / lookup / heartbeat TTL /
evict, persistence), fail-open client, durable queue with stale in-flight reclaim, and
the router's locality / transfer-vs-recompute decisions."""
import time

from axropus_deploy_b200.cluster import (AmfCoordinator, ClusterRouter, CoordinatorClient, InProcQueue,
                                         SqliteQueue, WorkerInfo, serve_coordinator)
from axropus_deploy_b200.cluster.router import amf_lookup_hash, canonicalize


def test_coordinator_http_roundtrip(tmp_path):
    db = str(tmp_path / "coord.db")
    coord = AmfCoordinator(db, node_ttl_s=30)
    srv, port = serve_coordinator(coord)
    try:
        c = CoordinatorClient(f"http://127.0.0.1:{port}", timeout_s=2.0)
        assert c.register("abc123", "node-a", "w0", "t1", {"tier": "g1_pool", "tokens": 8192})
        assert c.register("abc123", "node-b", "w5", "t1")
        locs = c.lookup("abc123", "t1")
        assert {l["node_id"] for l in locs} == {"node-a", "node-b"}
        assert c.lookup("abc123", "other-tenant") == []
        # heartbeat with an entry list replaces node-b's registrations
        assert c.heartbeat("node-b", [{"tenant_id": "t1", "prefix_hash": "ffff", "worker_id": "w5"}])
        assert {l["node_id"] for l in c.lookup("abc123", "t1")} == {"node-a"}
        assert c.evict("abc123", "t1") == 1
        assert c.lookup("abc123", "t1") == []
    finally:
        srv.shutdown()
    # persistence: a new coordinator on the same file still knows node-b's entry
    assert AmfCoordinator(db).lookup("t1", "ffff")[0]["worker_id"] == "w5"


def test_coordinator_node_ttl_and_fail_open():
    coord = AmfCoordinator(node_ttl_s=10)
    coord.register("t", "k1", "node-a", "w0", now=100.0)
    assert coord.lookup("t", "k1", now=105.0)
    assert coord.lookup("t", "k1", now=111.0) == []  # node-a missed its heartbeats
    coord.heartbeat("node-a", now=112.0)
    assert coord.lookup("t", "k1", now=113.0)
    dead = CoordinatorClient("http://127.0.0.1:9", timeout_s=0.1)  # nothing listens
    t0 = time.time()
    assert dead.lookup("k1") == [] and not dead.register("k1", "n") and dead.errors == 2
    assert time.time() - t0 < 2.0


def test_sqlite_queue_reclaims_stale(tmp_path):
    q = SqliteQueue(str(tmp_path / "q.db"), visibility_s=5)
    a = q.enqueue({"job": 1})
    q.enqueue({"job": 2}, delay_s=1000)
    iid, item = q.dequeue(now=time.time())
    assert iid == a and item == {"job": 1}
    assert q.dequeue() is None  # job 2 is delayed, job 1 in flight
    # the consumer died: after the visibility window job 1 is handed out again
    again = q.dequeue(now=time.time() + 10)
    assert again is not None and again[0] == a
    assert q.ack(a) and q.stats()["ready"] == 1
    iq = InProcQueue()
    i1 = iq.enqueue("x")
    iid, _ = iq.dequeue()
    assert iq.retry(iid) and iq.dequeue()[0] == i1 and iq.stats()["inflight"] == 1


def test_router_locality_transfer_and_cold():
    coord = AmfCoordinator()
    qa, qb = InProcQueue(), InProcQueue()
    wa = WorkerInfo("wa", "node-a", load=0, queue=qa)
    wb = WorkerInfo("wb", "node-b", load=0, spec=True, queue=qb)
    r = ClusterRouter([wa, wb], coord, prefix_tokens=64)
    prompt = "system: you are a helpful agent. " * 4
    first = r.submit(prompt, "t")
    assert first.kind == "cold" and first.lane.endswith("MISS")
    coord.register("t", first.prefix_key, first.worker.node_id, first.worker.worker_id)
    first.worker.load = 0  # the first request finished
    # same prefix: routed to the holder
    again = r.submit(prompt + " next turn", "t")
    assert again.kind == "amf_local" and again.worker is first.worker and again.lane.endswith("HIT")
    # holder overloaded: the other worker takes it; KV moves only if the link beats recompute
    first.worker.load += 10_000
    far = r.submit(prompt + " third", "t")
    assert far.worker is not first.worker and far.kind in ("amf_transfer", "recompute")
    assert (qa.stats()["ready"] + qb.stats()["ready"]) == 3
    assert canonicalize("a  \t b\n\n\n\nc ") == "a b\n\nc"
    assert amf_lookup_hash("t", "x") != amf_lookup_hash("u", "x")
