"""Networked work queues: Redis Streams, NATS and SQS, spoken directly on their wire
protocols (RESP2, the NATS text protocol, the SQS JSON API signed with SigV4) so that no
client library is needed. Same interface as the local queues: ``enqueue(item, delay_s) ->
id``, ``dequeue() -> (id, item) | None``, ``ack``, ``retry``, ``stats``.

* :class:`RedisStreamQueue` -- one stream per queue name and a consumer group. Delayed
  items wait in a sorted set scored by their ready time and move to the stream when due
  (``ZREM`` decides which consumer moves one). An entry a consumer took but neither acked
  nor retried within ``visibility_s`` is claimed by the next consumer (``XAUTOCLAIM``),
  the stale in-flight reclaim of the SQLite queue.
* :class:`NatsQueue` -- core NATS publish / queue-group subscribe: every item goes to one
  subscriber of the group; like the reference's it is not durable (ack is local, retry
  publishes again, delays are kept by the retrying consumer).
* :class:`SqsQueue` -- SendMessage / ReceiveMessage / DeleteMessage /
  ChangeMessageVisibility (retry = visibility ``delay_s``) / GetQueueAttributes.

:func:`build_queue` picks one from ``KORITH_QUEUE_BACKEND`` (``sqlite`` default, ``inproc``,
``redis`` / ``redis_streams`` with ``KORITH_REDIS_URL``, ``nats`` with ``KORITH_NATS_URL``,
``sqs`` with ``KORITH_SQS_URL``).

Reference: platform/queue/redis_queue.py, redis_streams.py, nats_queue.py, sqs_queue.py and
platform/runtime/config.py:152-171 (backend selection and its variables).
"""
from __future__ import annotations

import json
import os
import socket
import threading
import time
import urllib.parse
import uuid
from collections import deque
from typing import Any, Dict, List, Optional, Tuple

from .queues import InProcQueue, SqliteQueue
from .sigv4 import SignedHttp


# ---------------------------------------------------------------------------------- RESP2
class RedisError(RuntimeError):
    pass


class RespClient:
    """Minimal Redis client: one socket, RESP2 requests as arrays of bulk strings, replies
    parsed into str / bytes / int / list / None. ``redis://[user:password@]host:port/db``.
    A dropped connection is reopened and the call retried once, unless the call is
    marked non-idempotent (``retry=False``): a command the server may already have
    applied before the connection dropped (INCRBY, a script that writes) is then not
    sent twice; the error reaches the caller instead."""

    def __init__(self, url: str = "redis://127.0.0.1:6379/0", timeout_s: float = 10.0):
        u = urllib.parse.urlsplit(url)
        self.host, self.port = u.hostname or "127.0.0.1", u.port or 6379
        self.timeout_s = timeout_s
        self._mu = threading.Lock()
        self._sock: Optional[socket.socket] = None
        self._buf = b""
        self._user, self._password = u.username, u.password
        self._db = int((u.path or "/0").strip("/") or 0)

    def _connect(self) -> None:
        self._sock, self._buf = socket.create_connection((self.host, self.port), timeout=self.timeout_s), b""
        if self._password:
            self._call_locked(*(["AUTH", self._user, self._password] if self._user else ["AUTH", self._password]))
        if self._db:
            self._call_locked("SELECT", self._db)

    def close(self) -> None:
        with self._mu:
            if self._sock is not None:
                self._sock.close()
                self._sock = None

    def _fill(self, cond) -> None:
        while not cond():
            chunk = self._sock.recv(65536)
            if not chunk:
                raise ConnectionError("redis connection closed")
            self._buf += chunk

    def _read(self) -> Any:
        self._fill(lambda: b"\r\n" in self._buf)
        line, self._buf = self._buf.split(b"\r\n", 1)
        kind, rest = line[:1], line[1:]
        if kind == b"+":
            return rest.decode()
        if kind == b"-":
            return RedisError(rest.decode())
        if kind == b":":
            return int(rest)
        if kind == b"$":
            n = int(rest)
            if n < 0:
                return None
            self._fill(lambda: len(self._buf) >= n + 2)
            data, self._buf = self._buf[:n], self._buf[n + 2:]
            return data
        if kind == b"*":
            n = int(rest)
            return None if n < 0 else [self._read() for _ in range(n)]
        raise RedisError(f"unexpected reply {line[:32]!r}")

    def _call_locked(self, *args) -> Any:
        parts = [b"*%d\r\n" % len(args)]
        for a in args:
            b = a if isinstance(a, bytes) else str(a).encode("utf-8")
            parts.append(b"$%d\r\n%s\r\n" % (len(b), b))
        self._sock.sendall(b"".join(parts))
        r = self._read()
        if isinstance(r, RedisError):
            raise r
        return r

    def call(self, *args, retry: bool = True) -> Any:
        with self._mu:
            for attempt in (0, 1):
                sent = False
                try:
                    if self._sock is None:
                        self._connect()
                    sent = True
                    return self._call_locked(*args)
                except (ConnectionError, OSError):
                    if self._sock is not None:
                        self._sock.close()
                    self._sock = None
                    if attempt or (sent and not retry):
                        raise


def _s(x: Any) -> str:
    return x.decode("utf-8") if isinstance(x, (bytes, bytearray)) else str(x)


class RedisStreamQueue:
    def __init__(self, url: str = "redis://127.0.0.1:6379/0", name: str = "default", prefix: str = "korith:jobs",
                 group: str = "korith", consumer: Optional[str] = None, visibility_s: float = 900.0,
                 client: Optional[RespClient] = None):
        self.r = client or RespClient(url)
        self.stream = f"{prefix}:{name}"
        self.delayed = f"{prefix}:{name}:delayed"
        self.group = group
        self.consumer = consumer or f"{socket.gethostname()}-{os.getpid()}-{uuid.uuid4().hex[:6]}"
        self.visibility_ms = int(visibility_s * 1000)
        self._inflight: Dict[str, Tuple[str, Any]] = {}  # item id -> (stream entry id, item)
        self.stat = {"enqueued": 0, "acked": 0, "retried": 0, "reclaimed": 0}
        try:
            self.r.call("XGROUP", "CREATE", self.stream, self.group, "0", "MKSTREAM")
        except RedisError as e:
            if "BUSYGROUP" not in str(e):
                raise

    def _add(self, iid: str, item: Any) -> None:
        self.r.call("XADD", self.stream, "*", "id", iid, "body", json.dumps(item), "enqueued_at", f"{time.time():.6f}")

    def _delay(self, iid: str, item: Any, delay_s: float) -> None:
        self.r.call("ZADD", self.delayed, f"{time.time() + delay_s:.6f}", json.dumps({"id": iid, "item": item}))

    def enqueue(self, item: Any, delay_s: float = 0.0) -> str:
        iid = uuid.uuid4().hex
        if delay_s > 0:
            self._delay(iid, item, delay_s)
        else:
            self._add(iid, item)
        self.stat["enqueued"] += 1
        return iid

    def _promote_due(self) -> None:
        due = self.r.call("ZRANGEBYSCORE", self.delayed, "-inf", f"{time.time():.6f}", "LIMIT", 0, 32) or []
        for m in due:
            if self.r.call("ZREM", self.delayed, m) == 1:  # only the consumer whose ZREM removed it moves it
                d = json.loads(_s(m))
                self._add(d["id"], d["item"])

    def _take(self, entry: List[Any]) -> Tuple[str, Any]:
        eid, flat = _s(entry[0]), entry[1] or []
        f = {_s(flat[i]): _s(flat[i + 1]) for i in range(0, len(flat) - 1, 2)}
        item = json.loads(f.get("body", "null"))
        self._inflight[f["id"]] = (eid, item)
        return f["id"], item

    def dequeue(self) -> Optional[Tuple[str, Any]]:
        self._promote_due()
        got = self.r.call("XAUTOCLAIM", self.stream, self.group, self.consumer, self.visibility_ms, "0-0", "COUNT", 1)
        claimed = [e for e in (got[1] if got and len(got) > 1 else []) if e and e[1]]
        if claimed:
            self.stat["reclaimed"] += 1
            return self._take(claimed[0])
        resp = self.r.call("XREADGROUP", "GROUP", self.group, self.consumer, "COUNT", 1, "STREAMS", self.stream, ">")
        if not resp:
            return None
        entries = resp[0][1]
        return self._take(entries[0]) if entries else None

    def _drop(self, iid: str) -> Optional[Tuple[str, Any]]:
        got = self._inflight.pop(iid, None)
        if got is not None:
            self.r.call("XACK", self.stream, self.group, got[0])
            self.r.call("XDEL", self.stream, got[0])
        return got

    def ack(self, iid: str) -> bool:
        ok = self._drop(iid) is not None
        self.stat["acked"] += int(ok)
        return ok

    def retry(self, iid: str, delay_s: float = 0.0) -> bool:
        got = self._drop(iid)
        if got is None:
            return False
        if delay_s > 0:
            self._delay(iid, got[1], delay_s)
        else:
            self._add(iid, got[1])
        self.stat["retried"] += 1
        return True

    def stats(self) -> Dict[str, int]:
        total = int(self.r.call("XLEN", self.stream))
        pend = self.r.call("XPENDING", self.stream, self.group)
        inflight = int(pend[0]) if pend else 0
        return dict(self.stat, ready=total - inflight, inflight=inflight,
                    delayed=int(self.r.call("ZCARD", self.delayed)))


# ---------------------------------------------------------------------------------- NATS
class NatsClient:
    """Core NATS over one socket: CONNECT, PUB, SUB (with a queue group), PING / PONG; a
    reader thread files MSG payloads per subscription."""

    def __init__(self, url: str = "nats://127.0.0.1:4222", timeout_s: float = 10.0, name: str = "axropus"):
        u = urllib.parse.urlsplit(url)
        self._sock = socket.create_connection((u.hostname or "127.0.0.1", u.port or 4222), timeout=timeout_s)
        self._mu = threading.Lock()
        self._cv = threading.Condition()
        self._msgs: Dict[str, deque] = {}
        self._pongs = 0
        self._closed = False
        self._buf = b""
        self._sid = 0
        self._line()  # the server's INFO
        self._sock.settimeout(None)
        opts: Dict[str, Any] = {"verbose": False, "pedantic": False, "name": name, "lang": "python", "version": "1"}
        if u.username:
            opts["user"] = urllib.parse.unquote(u.username)
            if u.password:
                opts["pass"] = urllib.parse.unquote(u.password)
        self._send(b"CONNECT " + json.dumps(opts).encode() + b"\r\n")
        self._reader = threading.Thread(target=self._loop, daemon=True)
        self._reader.start()
        self.flush(timeout_s)

    def _send(self, data: bytes) -> None:
        with self._mu:
            self._sock.sendall(data)

    def _fill(self, cond) -> None:
        while not cond():
            chunk = self._sock.recv(65536)
            if not chunk:
                raise ConnectionError("nats connection closed")
            self._buf += chunk

    def _line(self) -> bytes:
        self._fill(lambda: b"\r\n" in self._buf)
        line, self._buf = self._buf.split(b"\r\n", 1)
        return line

    def _loop(self) -> None:
        try:
            while not self._closed:
                line = self._line()
                op = line.split(b" ", 1)[0].upper()
                if op == b"MSG":  # MSG <subject> <sid> [reply-to] <#bytes>
                    parts = line.split()
                    n = int(parts[-1])
                    self._fill(lambda: len(self._buf) >= n + 2)
                    data, self._buf = self._buf[:n], self._buf[n + 2:]
                    with self._cv:
                        self._msgs.setdefault(_s(parts[2]), deque()).append(data)
                        self._cv.notify_all()
                elif op == b"PING":
                    self._send(b"PONG\r\n")
                elif op == b"PONG":
                    with self._cv:
                        self._pongs += 1
                        self._cv.notify_all()
        except (OSError, ConnectionError, ValueError):
            pass
        with self._cv:
            self._closed = True
            self._cv.notify_all()

    def flush(self, timeout_s: float = 10.0) -> None:
        """Round trip to the server: everything sent before has been processed."""
        with self._cv:
            want = self._pongs + 1
        self._send(b"PING\r\n")
        with self._cv:
            self._cv.wait_for(lambda: self._pongs >= want or self._closed, timeout_s)
            if self._pongs < want:
                raise ConnectionError("nats server did not answer PING")

    def publish(self, subject: str, data: bytes) -> None:
        self._send(b"PUB %s %d\r\n%s\r\n" % (subject.encode(), len(data), data))

    def subscribe(self, subject: str, queue: str = "") -> str:
        self._sid += 1
        sid = str(self._sid)
        with self._cv:
            self._msgs[sid] = deque()
        self._send((f"SUB {subject} {queue} {sid}\r\n" if queue else f"SUB {subject} {sid}\r\n").encode())
        return sid

    def next_msg(self, sid: str, timeout_s: float = 0.0) -> Optional[bytes]:
        with self._cv:
            self._cv.wait_for(lambda: self._msgs.get(sid) or self._closed, timeout_s)
            q = self._msgs.get(sid)
            return q.popleft() if q else None

    def close(self) -> None:
        self._closed = True
        try:
            self._sock.shutdown(socket.SHUT_RDWR)
        except OSError:
            pass
        self._sock.close()


class NatsQueue:
    def __init__(self, url: str = "nats://127.0.0.1:4222", name: str = "default", subject_prefix: str = "korith.queue",
                 group: str = "korith", client: Optional[NatsClient] = None, wait_s: float = 0.0):
        self.nc = client or NatsClient(url)
        self.subject = f"{subject_prefix}.{name}"
        self.sid = self.nc.subscribe(self.subject, group)
        self.nc.flush()
        self.wait_s = wait_s
        self._inflight: Dict[str, Any] = {}
        self._delayed: List[Tuple[float, str, Any]] = []
        self.stat = {"enqueued": 0, "acked": 0, "retried": 0}

    def _pub(self, iid: str, item: Any) -> None:
        self.nc.publish(self.subject, json.dumps({"id": iid, "item": item, "enqueued_at": time.time()}).encode())

    def enqueue(self, item: Any, delay_s: float = 0.0) -> str:
        iid = uuid.uuid4().hex
        if delay_s > 0:
            self._delayed.append((time.monotonic() + delay_s, iid, item))
        else:
            self._pub(iid, item)
        self.stat["enqueued"] += 1
        return iid

    def dequeue(self) -> Optional[Tuple[str, Any]]:
        now = time.monotonic()
        for d in [d for d in self._delayed if d[0] <= now]:
            self._delayed.remove(d)
            self._pub(d[1], d[2])
        data = self.nc.next_msg(self.sid, self.wait_s)
        if data is None:
            return None
        env = json.loads(data)
        self._inflight[env["id"]] = env["item"]
        return env["id"], env["item"]

    def ack(self, iid: str) -> bool:
        ok = self._inflight.pop(iid, None) is not None
        self.stat["acked"] += int(ok)
        return ok

    def retry(self, iid: str, delay_s: float = 0.0) -> bool:
        if iid not in self._inflight:
            return False
        item = self._inflight.pop(iid)
        if delay_s > 0:
            self._delayed.append((time.monotonic() + delay_s, iid, item))
        else:
            self._pub(iid, item)
        self.stat["retried"] += 1
        return True

    def stats(self) -> Dict[str, int]:
        return dict(self.stat, inflight=len(self._inflight), delayed=len(self._delayed))


# ---------------------------------------------------------------------------------- SQS
class SqsQueue:
    """An SQS queue by its URL (``https://sqs.<region>.amazonaws.com/<account>/<name>`` or a
    compatible endpoint). Items travel as JSON message bodies."""

    def __init__(self, queue_url: str, region: Optional[str] = None, http: Optional[SignedHttp] = None,
                 wait_s: int = 0, visibility_s: int = 900):
        self.url = queue_url
        u = urllib.parse.urlsplit(queue_url)
        host = u.hostname or ""
        if region is None and host.startswith("sqs.") and host.count(".") >= 3:
            region = host.split(".")[1]
        self.http = http or SignedHttp("sqs", region)
        self.endpoint = f"{u.scheme}://{u.netloc}/"
        self.wait_s, self.visibility_s = int(wait_s), int(visibility_s)
        self._receipts: Dict[str, str] = {}
        self.stat = {"enqueued": 0, "acked": 0, "retried": 0}

    def _call(self, action: str, body: Dict[str, Any]) -> Dict[str, Any]:
        payload = json.dumps(dict(body, QueueUrl=self.url)).encode()
        st, _, out = self.http.request("POST", self.endpoint, payload,
                                       {"content-type": "application/x-amz-json-1.0",
                                        "x-amz-target": f"AmazonSQS.{action}"})
        if st != 200:
            raise RuntimeError(f"SQS {action} failed: HTTP {st} {out[:200]!r}")
        return json.loads(out or b"{}")

    def enqueue(self, item: Any, delay_s: float = 0.0) -> str:
        iid = uuid.uuid4().hex
        self._call("SendMessage", {"MessageBody": json.dumps({"id": iid, "item": item, "enqueued_at": time.time()}),
                                   "DelaySeconds": int(min(900, max(0, round(delay_s))))})
        self.stat["enqueued"] += 1
        return iid

    def dequeue(self) -> Optional[Tuple[str, Any]]:
        r = self._call("ReceiveMessage", {"MaxNumberOfMessages": 1, "WaitTimeSeconds": self.wait_s,
                                          "VisibilityTimeout": self.visibility_s})
        msgs = r.get("Messages") or []
        if not msgs:
            return None
        env = json.loads(msgs[0]["Body"])
        self._receipts[env["id"]] = msgs[0]["ReceiptHandle"]
        return env["id"], env["item"]

    def ack(self, iid: str) -> bool:
        rh = self._receipts.pop(iid, None)
        if rh is None:
            return False
        self._call("DeleteMessage", {"ReceiptHandle": rh})
        self.stat["acked"] += 1
        return True

    def retry(self, iid: str, delay_s: float = 0.0) -> bool:
        rh = self._receipts.pop(iid, None)
        if rh is None:
            return False
        self._call("ChangeMessageVisibility", {"ReceiptHandle": rh, "VisibilityTimeout": int(max(0, round(delay_s)))})
        self.stat["retried"] += 1
        return True

    def stats(self) -> Dict[str, int]:
        a = self._call("GetQueueAttributes", {"AttributeNames": ["ApproximateNumberOfMessages",
                                                                 "ApproximateNumberOfMessagesNotVisible"]})
        attrs = a.get("Attributes") or {}
        return dict(self.stat, ready=int(attrs.get("ApproximateNumberOfMessages", 0)),
                    inflight=int(attrs.get("ApproximateNumberOfMessagesNotVisible", 0)))


# ---------------------------------------------------------------------------------- selection
def build_queue(name: str = "default", backend: Optional[str] = None):
    """The queue ``KORITH_QUEUE_BACKEND`` names, for queue ``name`` (one per lane)."""
    b = (backend or os.environ.get("KORITH_QUEUE_BACKEND", "sqlite")).strip().lower()
    if b == "inproc":
        return InProcQueue()
    if b in ("redis", "redis_streams"):
        node = os.environ.get("KORITH_NODE_ID", "").strip()
        return RedisStreamQueue(os.environ.get("KORITH_REDIS_URL", "redis://127.0.0.1:6379/0"),
                                name=f"{node}:{name}" if (b == "redis_streams" and node) else name,
                                prefix=os.environ.get("KORITH_STREAM_PREFIX", "korith:jobs"),
                                group=os.environ.get("KORITH_STREAM_CONSUMER_GROUP", "korith"),
                                visibility_s=float(os.environ.get("KORITH_QUEUE_INFLIGHT_STALE_S", "900")))
    if b == "nats":
        return NatsQueue(os.environ.get("KORITH_NATS_URL", "nats://127.0.0.1:4222"), name=name)
    if b == "sqs":
        url = os.environ.get("KORITH_SQS_URL", "")
        if not url:
            raise ValueError("KORITH_QUEUE_BACKEND=sqs needs KORITH_SQS_URL")
        return SqsQueue(url.replace("{lane}", name))
    if b != "sqlite":
        raise ValueError(f"unknown KORITH_QUEUE_BACKEND {b!r}")
    path = os.environ.get("KORITH_QUEUE_DB", "./platform_data/queue.sqlite")
    if path != ":memory:":
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    return SqliteQueue(path, name=name, visibility_s=float(os.environ.get("KORITH_QUEUE_INFLIGHT_STALE_S", "900")))
