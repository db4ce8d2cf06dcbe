"""Networked queues and the S3 / MinIO artifact store against in-process fake servers that
speak the real wire protocols: RESP2 (Redis streams, consumer groups, XAUTOCLAIM, sorted
sets), the NATS text protocol (queue groups) and S3 / SQS over HTTP, where the fake
re-derives every request's SigV4 signature and refuses a mismatch. SigV4 itself is checked
against AWS's published example values.

Reference: platform/tests/test_queue.py (enqueue / dequeue / ack / retry / reclaim) and the
S3 / MinIO adapters of platform/artifacts.
"""
import datetime as dt
import json
import socketserver
import threading
import time
import urllib.parse
from collections import OrderedDict
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import pytest

from axropus_deploy_b200.cluster import netqueues as nq
from axropus_deploy_b200.cluster.objstore import S3ArtifactStore, build_artifacts, LocalArtifactStore
from axropus_deploy_b200.cluster.sigv4 import Credentials, SignedHttp, sign, signing_key

SECRET = "test-secret-key"
CREDS = Credentials("AKTEST", SECRET)


# ----------------------------------------------------------------------------- SigV4
def test_sigv4_published_examples():
    # AWS's documented derived key (iam, 20120215) and the get-vanilla request signature
    k = signing_key("wJalrXUtnFEMI/K7MDENG+bPxRfiCYEXAMPLEKEY", "20120215", "us-east-1", "iam")
    assert k.hex() == "f4780e2d9f65fa895f9c67b32ce1baf0b0d8a43505a000a1a9e090d414db404d"
    h = sign("GET", "https://example.amazonaws.com/", {}, b"",
             Credentials("AKIDEXAMPLE", "wJalrXUtnFEMI/K7MDENG+bPxRfiCYEXAMPLEKEY"), "us-east-1", "service",
             now=dt.datetime(2015, 8, 30, 12, 36, 0))
    assert h["Authorization"].endswith("SignedHeaders=host;x-amz-date, "
                                       "Signature=5fa00fa31553b73ebf1942676e86291e8372ff2a2260956d9b8aae1d763fbf31")


# ----------------------------------------------------------------------------- fake Redis
class _FakeRedis:
    def __init__(self, password=None):
        self.mu = threading.Lock()
        self.streams = {}
        self.zsets = {}
        self.seq = 0
        self.password = password

    @staticmethod
    def _id(s):
        a, b = s.split("-")
        return int(a), int(b)

    def do(self, conn, args):
        cmd = args[0].upper()
        a = args[1:]
        if self.password and not conn.get("auth") and cmd != "AUTH":
            return Exception("NOAUTH Authentication required.")
        if cmd == "AUTH":
            if a[-1] != self.password:
                return Exception("WRONGPASS invalid password")
            conn["auth"] = True
            return "+OK"
        if cmd in ("PING", "SELECT"):
            return "+OK"
        if cmd == "XGROUP":
            st = self.streams.setdefault(a[1], {"entries": OrderedDict(), "groups": {}})
            if a[2] in st["groups"]:
                return Exception("BUSYGROUP Consumer Group name already exists")
            st["groups"][a[2]] = {"last": (0, 0), "pending": {}}
            return "+OK"
        if cmd == "XADD":
            st = self.streams.setdefault(a[0], {"entries": OrderedDict(), "groups": {}})
            self.seq += 1
            eid = f"{int(time.time() * 1000)}-{self.seq}"
            st["entries"][eid] = list(a[2:])
            return eid.encode()
        if cmd == "XREADGROUP":  # GROUP g c COUNT n STREAMS key >
            g, c, n, key = a[1], a[2], int(a[4]), a[6]
            st, grp = self.streams[key], self.streams[key]["groups"][g]
            out = []
            for eid, f in st["entries"].items():
                if self._id(eid) > grp["last"] and len(out) < n:
                    grp["last"] = self._id(eid)
                    grp["pending"][eid] = [c, time.time() * 1000]
                    out.append([eid.encode(), [x.encode() for x in f]])
            return [[key.encode(), out]] if out else None
        if cmd == "XAUTOCLAIM":  # key group consumer min-idle start COUNT n
            key, g, c, idle, n = a[0], a[1], a[2], float(a[3]), int(a[6])
            st, grp = self.streams[key], self.streams[key]["groups"][a[1]]
            now, got, deleted = time.time() * 1000, [], []
            for eid in sorted(grp["pending"], key=self._id):
                if len(got) >= n:
                    break
                if now - grp["pending"][eid][1] >= idle:
                    if eid not in st["entries"]:
                        del grp["pending"][eid]
                        deleted.append(eid.encode())
                        continue
                    grp["pending"][eid] = [c, now]
                    got.append([eid.encode(), [x.encode() for x in st["entries"][eid]]])
            return [b"0-0", got, deleted]
        if cmd == "XACK":
            grp = self.streams[a[0]]["groups"][a[1]]
            return sum(1 for e in a[2:] if grp["pending"].pop(e, None) is not None)
        if cmd == "XDEL":
            return sum(1 for e in a[1:] if self.streams[a[0]]["entries"].pop(e, None) is not None)
        if cmd == "XLEN":
            return len(self.streams.get(a[0], {"entries": {}})["entries"])
        if cmd == "XPENDING":
            p = self.streams[a[0]]["groups"][a[1]]["pending"]
            return [len(p), None, None, None]
        if cmd == "ZADD":
            self.zsets.setdefault(a[0], {})[a[2]] = float(a[1])
            return 1
        if cmd == "ZRANGEBYSCORE":
            z = self.zsets.get(a[0], {})
            hi = float(a[2])
            ms = sorted((s, m) for m, s in z.items() if s <= hi)
            off, cnt = (int(a[4]), int(a[5])) if len(a) > 3 else (0, len(ms))
            return [m.encode() for _, m in ms[off:off + cnt]]
        if cmd == "ZREM":
            return 1 if self.zsets.get(a[0], {}).pop(a[1], None) is not None else 0
        if cmd == "ZCARD":
            return len(self.zsets.get(a[0], {}))
        kv = self.__dict__.setdefault("kv", {})
        if cmd == "SET":
            kv[a[0]] = a[1]
            return "+OK"
        if cmd == "GET":
            v = kv.get(a[0])
            return v if isinstance(v, str) else None
        if cmd == "DEL":
            return 1 if kv.pop(a[0], None) is not None else 0
        if cmd == "SADD":
            st = kv.setdefault(a[0], set())
            n = sum(1 for m in a[1:] if m not in st)
            st.update(a[1:])
            return n
        if cmd == "SMEMBERS":
            return sorted(kv.get(a[0], set()))
        if cmd == "HSET":
            h = kv.setdefault(a[0], {})
            for i in range(1, len(a) - 1, 2):
                h[a[i]] = a[i + 1]
            return len(a) // 2
        if cmd == "HGETALL":
            return [x for k, v in kv.get(a[0], {}).items() for x in (k, v)]
        if cmd in ("INCRBY", "DECRBY"):
            n = int(kv.get(a[0], 0)) + (int(a[1]) if cmd == "INCRBY" else -int(a[1]))
            kv[a[0]] = n
            return n
        if cmd == "EXPIRE":
            return 1
        if cmd == "EVAL":
            # no Lua here: the fake knows the one script the gateway sends and runs its
            # semantics (check both windows, then consume) under the server lock
            from axropus_deploy_b200.cluster.gateway import RATE_LIMIT_LUA

            if a[0] != RATE_LIMIT_LUA:
                return Exception("ERR unknown script")
            rk, tk, rcap, tcap, toks = a[2], a[3], int(a[4]), int(a[5]), int(a[6])
            r, t = int(kv.get(rk, 0)), int(kv.get(tk, 0))
            if r + 1 > rcap:
                return [0, 1]
            if t + toks > tcap:
                return [0, 2]
            kv[rk], kv[tk] = r + 1, t + toks
            return [1, 0]
        return Exception(f"ERR unknown command {cmd}")

    @staticmethod
    def enc(x):
        if isinstance(x, Exception):
            return b"-" + str(x).encode() + b"\r\n"
        if x is None:
            return b"$-1\r\n"
        if isinstance(x, str) and x.startswith("+"):
            return x.encode() + b"\r\n"
        if isinstance(x, int):
            return b":%d\r\n" % x
        if isinstance(x, (bytes, str)):
            b = x if isinstance(x, bytes) else x.encode()
            return b"$%d\r\n%s\r\n" % (len(b), b)
        return b"*%d\r\n" % len(x) + b"".join(_FakeRedis.enc(v) for v in x)

    def serve(self):
        fake = self

        class H(socketserver.StreamRequestHandler):
            def handle(self):
                conn = {}
                while True:
                    line = self.rfile.readline()
                    if not line:
                        return
                    n = int(line[1:])
                    args = []
                    for _ in range(n):
                        ln = int(self.rfile.readline()[1:])
                        args.append(self.rfile.read(ln + 2)[:-2].decode())
                    with fake.mu:
                        r = fake.do(conn, args)
                    self.wfile.write(fake.enc(r))

        srv = socketserver.ThreadingTCPServer(("127.0.0.1", 0), H)
        srv.daemon_threads = True
        threading.Thread(target=srv.serve_forever, daemon=True).start()
        return srv


@pytest.fixture
def redis_url():
    srv = _FakeRedis(password="pw").serve()
    yield f"redis://:pw@127.0.0.1:{srv.server_address[1]}/0"
    srv.shutdown()
    srv.server_close()


def test_redis_stream_queue_order_ack_retry(redis_url):
    q = nq.RedisStreamQueue(redis_url, name="HIT", consumer="w0")
    ids = [q.enqueue({"job": i}) for i in range(3)]
    got = [q.dequeue() for _ in range(3)]
    assert [g[0] for g in got] == ids and [g[1]["job"] for g in got] == [0, 1, 2]
    assert q.dequeue() is None
    assert q.stats()["inflight"] == 3
    assert q.ack(ids[0]) and not q.ack(ids[0])
    assert q.retry(ids[1], delay_s=0.2)
    assert q.retry(ids[2])
    assert q.dequeue() == (ids[2], {"job": 2})  # retried without delay: ready again
    assert q.dequeue() is None                   # the delayed one is not due yet
    assert q.stats()["delayed"] == 1
    time.sleep(0.25)
    assert q.dequeue() == (ids[1], {"job": 1})
    q.ack(ids[1])
    q.ack(ids[2])
    s = q.stats()
    assert (s["ready"], s["inflight"], s["delayed"]) == (0, 0, 0)


def test_redis_stream_queue_reclaims_stale_inflight(redis_url):
    a = nq.RedisStreamQueue(redis_url, name="MISS", consumer="a", visibility_s=0.1)
    b = nq.RedisStreamQueue(redis_url, name="MISS", consumer="b", visibility_s=0.1)
    iid = a.enqueue({"job": "x"})
    assert a.dequeue() == (iid, {"job": "x"})    # a takes it, then vanishes without ack
    assert b.dequeue() is None
    time.sleep(0.15)
    assert b.dequeue() == (iid, {"job": "x"})
    assert b.stat["reclaimed"] == 1 and b.ack(iid)
    assert b.dequeue() is None


def test_redis_wrong_password_refused(redis_url):
    bad = redis_url.replace(":pw@", ":nope@")
    with pytest.raises(nq.RedisError):
        nq.RedisStreamQueue(bad, name="X")


def test_build_queue_backends(redis_url, monkeypatch, tmp_path):
    monkeypatch.setenv("KORITH_QUEUE_BACKEND", "redis_streams")
    monkeypatch.setenv("KORITH_REDIS_URL", redis_url)
    monkeypatch.setenv("KORITH_NODE_ID", "node7")
    q = nq.build_queue("HIT")
    assert isinstance(q, nq.RedisStreamQueue) and q.stream == "korith:jobs:node7:HIT"
    monkeypatch.setenv("KORITH_QUEUE_BACKEND", "sqlite")
    monkeypatch.setenv("KORITH_QUEUE_DB", str(tmp_path / "q" / "queue.sqlite"))
    q = nq.build_queue("MISS")
    iid = q.enqueue({"a": 1})
    assert q.dequeue() == (iid, {"a": 1})
    monkeypatch.setenv("KORITH_QUEUE_BACKEND", "bogus")
    with pytest.raises(ValueError):
        nq.build_queue()


# ----------------------------------------------------------------------------- fake NATS
def _fake_nats():
    subs = []  # (conn, subject, queue, sid)
    mu = threading.Lock()
    rr = {}

    class H(socketserver.StreamRequestHandler):
        def handle(self):
            self.wlock = threading.Lock()
            self.send(b'INFO {"server_id":"fake","max_payload":1048576}\r\n')
            while True:
                line = self.rfile.readline()
                if not line:
                    break
                parts = line.decode().strip().split()
                if not parts:
                    continue
                op = parts[0].upper()
                if op == "PING":
                    self.send(b"PONG\r\n")
                elif op == "SUB":
                    subj, sid = parts[1], parts[-1]
                    queue = parts[2] if len(parts) == 4 else ""
                    with mu:
                        subs.append((self, subj, queue, sid))
                elif op == "PUB":
                    subj, n = parts[1], int(parts[-1])
                    data = self.rfile.read(n + 2)[:-2]
                    with mu:
                        targets = [s for s in subs if s[1] == subj]
                        plain = [s for s in targets if not s[2]]
                        groups = {}
                        for s in targets:
                            if s[2]:
                                groups.setdefault(s[2], []).append(s)
                        for g, members in groups.items():
                            k = rr.get((subj, g), 0)
                            rr[(subj, g)] = k + 1
                            plain.append(members[k % len(members)])
                    for c, _, _, sid in plain:
                        c.send(b"MSG %s %s %d\r\n%s\r\n" % (subj.encode(), sid.encode(), len(data), data))
            with mu:
                subs[:] = [s for s in subs if s[0] is not self]

        def send(self, b):
            with self.wlock:
                self.wfile.write(b)
                self.wfile.flush()

    srv = socketserver.ThreadingTCPServer(("127.0.0.1", 0), H)
    srv.daemon_threads = True
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv


def test_nats_queue_group_delivers_each_item_once():
    srv = _fake_nats()
    url = f"nats://127.0.0.1:{srv.server_address[1]}"
    try:
        a, b = nq.NatsQueue(url, name="HIT"), nq.NatsQueue(url, name="HIT")
        ids = {a.enqueue({"n": i}) for i in range(6)}
        a.nc.flush()
        got = {}
        deadline = time.time() + 5
        while len(got) < 6 and time.time() < deadline:
            for q in (a, b):
                r = q.dequeue()
                if r:
                    assert r[0] not in got
                    got[r[0]] = q
        assert set(got) == ids
        assert {id(q) for q in got.values()} == {id(a), id(b)}  # the group spread the items
        one = next(iter(got))
        owner = got[one]
        assert owner.retry(one) and owner.nc.flush() is None
        again = None
        deadline = time.time() + 5
        while again is None and time.time() < deadline:
            again = a.dequeue() or b.dequeue()
        assert again is not None and again[0] == one
        a.nc.close()
        b.nc.close()
    finally:
        srv.shutdown()
        srv.server_close()


# ----------------------------------------------------------------------------- fake S3 / SQS
def _signed_ok(handler, body):
    auth = handler.headers.get("Authorization", "")
    svc = auth.split("Credential=")[1].split(",")[0].split("/")[3]
    region = auth.split("Credential=")[1].split(",")[0].split("/")[2]
    signed = auth.split("SignedHeaders=")[1].split(",")[0].split(";")
    hdrs = {k: handler.headers[k] for k in signed if k not in ("host", "x-amz-date", "x-amz-content-sha256",
                                                                "x-amz-security-token")}
    url = f"http://{handler.headers['host']}{handler.path}"
    when = dt.datetime.strptime(handler.headers["x-amz-date"], "%Y%m%dT%H%M%SZ")
    want = sign(handler.command, url, hdrs, body, CREDS, region, svc, now=when)["Authorization"]
    return want == auth


def _fake_http(state):
    class H(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def _body(self):
            n = int(self.headers.get("Content-Length") or 0)
            return self.rfile.read(n) if n else b""

        def _reply(self, st, body=b"", ctype="application/xml"):
            self.send_response(st)
            self.send_header("Content-Type", ctype)
            self.send_header("Content-Length", str(len(body)))
            self.end_headers()
            self.wfile.write(body)

        def _handle(self):
            body = self._body()
            if not _signed_ok(self, body):
                state["rejected"] += 1
                return self._reply(403, b"<Error><Code>SignatureDoesNotMatch</Code></Error>")
            if self.headers.get("x-amz-target"):
                return self._sqs(self.headers["x-amz-target"].split(".")[1], json.loads(body))
            u = urllib.parse.urlsplit(self.path)
            bucket, _, key = u.path.lstrip("/").partition("/")
            key = urllib.parse.unquote(key)
            objs = state["s3"].setdefault(bucket, {})
            if self.command == "PUT":
                objs[key] = body
                return self._reply(200)
            if self.command == "DELETE":
                objs.pop(key, None)
                return self._reply(204)
            if key:
                return self._reply(200, objs[key], "application/octet-stream") if key in objs else self._reply(404)
            q = dict(urllib.parse.parse_qsl(u.query))
            keys = sorted(k for k in objs if k.startswith(q.get("prefix", "")))
            start = int(q.get("continuation-token", 0))
            page = keys[start:start + 2]
            more = start + 2 < len(keys)
            xml = ('<ListBucketResult xmlns="http://s3.amazonaws.com/doc/2006-03-01/">'
                   + "".join(f"<Contents><Key>{k}</Key></Contents>" for k in page)
                   + f"<IsTruncated>{'true' if more else 'false'}</IsTruncated>"
                   + (f"<NextContinuationToken>{start + 2}</NextContinuationToken>" if more else "")
                   + "</ListBucketResult>")
            return self._reply(200, xml.encode())

        def _sqs(self, action, req):
            msgs, now = state["sqs"], time.time()
            out = {}
            if action == "SendMessage":
                state["n"] += 1
                msgs.append({"Body": req["MessageBody"], "rh": f"rh{state['n']}",
                             "visible_at": now + req.get("DelaySeconds", 0)})
            elif action == "ReceiveMessage":
                for m in msgs:
                    if m["visible_at"] <= now:
                        m["visible_at"] = now + req["VisibilityTimeout"]
                        out = {"Messages": [{"Body": m["Body"], "ReceiptHandle": m["rh"]}]}
                        break
            elif action == "DeleteMessage":
                msgs[:] = [m for m in msgs if m["rh"] != req["ReceiptHandle"]]
            elif action == "ChangeMessageVisibility":
                for m in msgs:
                    if m["rh"] == req["ReceiptHandle"]:
                        m["visible_at"] = now + req["VisibilityTimeout"]
            elif action == "GetQueueAttributes":
                vis = sum(1 for m in msgs if m["visible_at"] <= now)
                out = {"Attributes": {"ApproximateNumberOfMessages": str(vis),
                                      "ApproximateNumberOfMessagesNotVisible": str(len(msgs) - vis)}}
            return self._reply(200, json.dumps(out).encode(), "application/x-amz-json-1.0")

        do_GET = do_PUT = do_POST = do_DELETE = _handle

    srv = ThreadingHTTPServer(("127.0.0.1", 0), H)
    srv.daemon_threads = True
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv


@pytest.fixture
def http_fake():
    state = {"s3": {}, "sqs": [], "n": 0, "rejected": 0}
    srv = _fake_http(state)
    yield f"http://127.0.0.1:{srv.server_address[1]}", state
    srv.shutdown()
    srv.server_close()


def test_s3_store_roundtrip_list_and_upload(http_fake, tmp_path):
    ep, state = http_fake
    st = S3ArtifactStore(tmp_path, "bucket", "korith", endpoint=ep, creds=CREDS)
    key = st.store_artifact("job 1", "output", b"hello world", org_id="acme")
    assert key == "korith/acme/job 1/output" and state["s3"]["bucket"][key] == b"hello world"
    assert st.get_artifact("job 1", "output", org_id="acme") == b"hello world"
    assert st.get_artifact("job 1", "log", org_id="acme") is None
    paths = st.init_job("job 1", "acme")
    paths["metrics"].write_text('{"ttft_ms": 7.1}')
    paths["log"].write_text("run log")
    assert sorted(st.upload_job("job 1", "acme")) == ["korith/acme/job 1/log", "korith/acme/job 1/metrics"]
    assert st.list_artifacts("job 1", "acme") == ["log", "metrics", "output"]  # over two list pages
    assert st.delete_artifact("job 1", "output", "acme") and st.get_artifact("job 1", "output", "acme") is None
    assert state["rejected"] == 0
    wrong = S3ArtifactStore(tmp_path, "bucket", endpoint=ep, creds=Credentials("AKTEST", "other"))
    with pytest.raises(RuntimeError):
        wrong.store_artifact("j", "output", b"x")
    assert state["rejected"] == 1


def test_build_artifacts_minio_and_local(http_fake, tmp_path, monkeypatch):
    ep, state = http_fake
    monkeypatch.setenv("KORITH_PLATFORM_ARTIFACTS", str(tmp_path))
    monkeypatch.setenv("KORITH_ARTIFACT_BACKEND", "minio")
    monkeypatch.setenv("KORITH_MINIO_ENDPOINT", ep.replace("http://", ""))
    monkeypatch.setenv("KORITH_MINIO_SECURE", "false")
    monkeypatch.setenv("KORITH_MINIO_ACCESS_KEY", "AKTEST")
    monkeypatch.setenv("KORITH_MINIO_SECRET_KEY", SECRET)
    monkeypatch.setenv("KORITH_MINIO_BUCKET", "art")
    st = build_artifacts()
    st.store_artifact("j", "events", b"{}\n")
    assert state["s3"]["art"]["korith/default/j/events"] == b"{}\n"
    monkeypatch.setenv("KORITH_ARTIFACT_BACKEND", "local")
    loc = build_artifacts()
    assert isinstance(loc, LocalArtifactStore)
    loc.store_artifact("j", "output", b"out")
    assert loc.get_artifact("j", "output") == b"out"


def test_sqs_queue_over_signed_json_api(http_fake):
    ep, state = http_fake
    q = nq.SqsQueue(f"{ep}/123456789012/korith-hit", http=SignedHttp("sqs", "us-west-2", CREDS))
    a = q.enqueue({"job": "a"})
    b = q.enqueue({"job": "b"})
    assert q.dequeue() == (a, {"job": "a"})
    assert q.dequeue() == (b, {"job": "b"})
    assert q.dequeue() is None
    assert q.stats()["inflight"] == 2
    assert q.ack(a)
    assert q.retry(b, delay_s=0)                 # visible again at once
    assert q.dequeue() == (b, {"job": "b"}) and q.ack(b)
    assert q.stats()["ready"] == 0 and state["sqs"] == [] and state["rejected"] == 0


def test_node_registry_and_snapshot_index_share_redis(redis_url, tmp_path):
    from axropus_deploy_b200.cluster.ledger import SqliteLedger
    from axropus_deploy_b200.cluster.nodes import NodeRegistry, SnapshotIndex

    # two nodes with separate SQLite files see each other through the Redis mirror
    a = NodeRegistry(str(tmp_path / "a.db"), redis_url=redis_url)
    b = NodeRegistry(str(tmp_path / "b.db"), redis_url=redis_url)
    a.register_or_heartbeat("node-a", "10.0.0.1", 9000, 8, inflight=2, capabilities={"gpu": "B200"})
    b.register_or_heartbeat("node-b", "10.0.0.2", 9000, 8)
    seen = a.list_nodes()
    assert [n["node_id"] for n in seen] == ["node-a", "node-b"] and seen[0]["capabilities"] == {"gpu": "B200"}
    assert b.get_node("node-a")["inflight"] == 2
    ia = SnapshotIndex(SqliteLedger(str(tmp_path / "la.db")), tier_roots={}, redis_url=redis_url)
    ib = SnapshotIndex(SqliteLedger(str(tmp_path / "lb.db")), tier_roots={}, redis_url=redis_url)
    ia.upsert_location("fp", "s1", "default", "node-a", "w0", "/x/vram/s1.amfk", 1234)
    locs = ib.get_locations("fp", "default")
    assert [(r["node_id"], r["snapshot_id"], r["storage_tier"]) for r in locs] == [("node-a", "s1", "vram")]
    # no Redis: the local copies still answer
    lone = NodeRegistry(str(tmp_path / "c.db"), redis_url="redis://127.0.0.1:1/0")
    assert lone.redis is None
    lone.register_or_heartbeat("node-c", "h", 1, 1)
    assert [n["node_id"] for n in lone.list_nodes()] == ["node-c"]


def test_deploy_config_reaches_the_environment(monkeypatch, capsys):
    import os

    from axropus_deploy_b200.cluster.__main__ import main

    saved = dict(os.environ)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    try:
        for k in [k for k in os.environ if k.startswith("KORITH_")]:
            del os.environ[k]
        os.environ["KORITH_CONFIG"] = os.path.join(root, "deploy", "config", "config.yaml")
        os.environ["KORITH_QUEUE_BACKEND"] = "inproc"  # set variables win over the file
        assert main(["apply-config", os.environ["KORITH_CONFIG"]]) == 0
        assert os.environ["KORITH_STREAM_PREFIX"] == "korith:jobs" and os.environ["KORITH_LEDGER_BACKEND"] == "sqlite"
        assert os.environ["KORITH_QUEUE_BACKEND"] == "inproc"
        assert os.environ["KORITH_NODE_REGISTRY_REDIS_URL"] == "redis://redis:6379/0"
    finally:
        os.environ.clear()
        os.environ.update(saved)


def test_deploy_rules_and_dashboard_name_exported_metrics():
    import os
    import re

    from axropus_deploy_b200.server.metrics import MetricRegistry as Metrics

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    obs = os.path.join(root, "deploy", "observability")
    text = open(os.path.join(obs, "alerts.yml")).read() + open(os.path.join(obs, "grafana-axropus-b200.json")).read()
    m = Metrics()
    if m.registry is None:
        pytest.skip("prometheus_client not installed")
    m.observe_request("g1_raw", 7.0, 4096)
    m.observe_request("cold", 120.0, 0)
    rendered = m.render().decode()
    src = "".join(open(os.path.join(root, "axropus_deploy_b200", "cluster", f)).read()
                  for f in os.listdir(os.path.join(root, "axropus_deploy_b200", "cluster")) if f.endswith(".py"))
    for name in sorted(set(re.findall(r"\b((?:axropus|korith)_[a-z_]+)", text))):
        if name.startswith("axropus_"):
            family = re.sub(r"_(total|sum|count)$", "", name)
            assert (re.search(rf"^{name}[{{ ]", rendered, re.M) or f"# TYPE {name} " in rendered
                    or f"# TYPE {family} " in rendered), name
        else:
            assert f'"{name}"' in src, name


def test_deploy_files_parse_and_agree():
    import os

    import yaml

    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "deploy")
    comp = yaml.safe_load(open(os.path.join(root, "docker-compose.yml")))
    assert comp["services"]["node-b"]["image"] == comp["services"]["node-a"]["image"] == "axropus-b200:latest"
    chart = os.path.join(root, "helm", "axropus-b200")
    assert yaml.safe_load(open(os.path.join(chart, "Chart.yaml")))["name"] == "axropus-b200"
    assert yaml.safe_load(open(os.path.join(chart, "values.yaml")))["nodes"]["gpusPerNode"] == 8
    # the chart carries its own copy of the platform config (Helm reads files inside the chart only)
    assert open(os.path.join(chart, "files", "config.yaml")).read() == open(os.path.join(root, "config",
                                                                                           "config.yaml")).read()


def test_worker_uploads_job_files_to_object_store(http_fake, tmp_path):
    import importlib.util
    import os

    from axropus_deploy_b200.cluster.objstore import S3ArtifactStore

    ep, state = http_fake
    here = os.path.dirname(os.path.abspath(__file__))
    spec = importlib.util.spec_from_file_location("platform_cpu", os.path.join(here, "test_platform_cpu.py"))
    pc = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(pc)
    plane, w, _ = pc._plane(tmp_path)
    w.uploader = S3ArtifactStore(w.artifacts.base, "jobs", "korith", endpoint=ep, creds=CREDS)
    jid = plane.submit({"prompt": "hello there", "max_tokens": 2}, org_id="org1")
    assert w.drain()[0]["exit_code"] == 0
    keys = sorted(state["s3"]["jobs"])
    assert f"korith/org1/{jid}/metrics" in keys and f"korith/org1/{jid}/output" in keys
    assert state["rejected"] == 0

    class Broken:
        def upload_job(self, *a):
            raise OSError("bucket unreachable")

    w.uploader = Broken()
    jid2 = plane.submit({"prompt": "hello again", "max_tokens": 2}, org_id="org1")
    assert w.drain()[0]["exit_code"] == 0 and plane.get_job(jid2, "org1")["status"] == "succeeded"
    assert any('status="failed"' in k for k in w.metrics.counters if k.startswith("korith_artifact_uploads_total"))


def test_gateway_rate_limit_shared_in_redis(redis_url, monkeypatch):
    from axropus_deploy_b200.cluster.gateway import RateLimiter

    monkeypatch.setenv("KORITH_RATE_LIMIT_BACKEND", "redis")
    monkeypatch.setenv("KORITH_REDIS_URL", redis_url)
    g1, g2 = RateLimiter(burst_factor=1.0), RateLimiter(burst_factor=1.0)  # two gateways, one budget
    now = 1_800_000_000.0
    got = [g.check_and_consume("acme", 10, rpm=3, tpm=1000, now=now)["allowed"] for g in (g1, g2, g1, g2)]
    assert got == [True, True, True, False]
    assert g1.check_and_consume("acme", 10, rpm=3, tpm=1000, now=now + 60)["allowed"]  # next window
    assert g2.check_and_consume("beta", 900, rpm=10, tpm=1000, now=now)["allowed"]
    r = g1.check_and_consume("beta", 200, rpm=10, tpm=1000, now=now)
    assert not r["allowed"] and r["reason"] == "tpm_exceeded"
    assert g2.check_and_consume("beta", 100, rpm=10, tpm=1000, now=now)["allowed"]  # the refusal used no quota


def test_resp_client_does_not_resend_non_idempotent_calls():
    from axropus_deploy_b200.cluster import netqueues as nq2

    c = nq2.RespClient("redis://127.0.0.1:1/0")
    sent = []

    def fake_connect():
        c._sock = type("S", (), {"close": lambda self: None})()

    def fake_call(*args):
        sent.append(args)
        raise ConnectionError("dropped after send")

    c._connect, c._call_locked = fake_connect, fake_call
    with pytest.raises(ConnectionError):
        c.call("INCRBY", "k", 1, retry=False)
    assert len(sent) == 1  # not sent a second time
    sent.clear()
    with pytest.raises(ConnectionError):
        c.call("GET", "k")
    assert len(sent) == 2  # idempotent: retried once
