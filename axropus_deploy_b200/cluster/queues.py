"""Work queues of the control plane: ``enqueue / dequeue / ack / retry / stats``.

:class:`InProcQueue` is a thread-safe in-memory queue; :class:`SqliteQueue` is durable
(one SQLite file, WAL) and reclaims in-flight items whose consumer vanished: an item
dequeued but neither acked nor retried within ``visibility_s`` becomes ready again.

Reference: platform/queue/base.py:15-29 (the interface) and platform/queue/sqlite_queue.py
(stale in-flight reclaim, :46-60).
"""
from __future__ import annotations

import json
import sqlite3
import threading
import time
import uuid
from collections import deque
from typing import Any, Dict, Optional, Tuple


class InProcQueue:
    def __init__(self):
        self._q: deque = deque()
        self._delayed: list = []
        self._inflight: Dict[str, Any] = {}
        self._mu = threading.Lock()
        self.stat = {"enqueued": 0, "acked": 0, "retried": 0}

    def enqueue(self, item: Any, delay_s: float = 0.0) -> str:
        iid = uuid.uuid4().hex
        with self._mu:
            if delay_s > 0:
                self._delayed.append((time.monotonic() + delay_s, iid, item))
            else:
                self._q.append((iid, item))
            self.stat["enqueued"] += 1
        return iid

    def dequeue(self) -> Optional[Tuple[str, Any]]:
        with self._mu:
            now = time.monotonic()
            ready = [d for d in self._delayed if d[0] <= now]
            for d in ready:
                self._delayed.remove(d)
                self._q.append((d[1], d[2]))
            if not self._q:
                return None
            iid, item = self._q.popleft()
            self._inflight[iid] = item
            return iid, item

    def ack(self, iid: str) -> bool:
        with self._mu:
            self.stat["acked"] += 1 if self._inflight.pop(iid, None) is not None else 0
            return True

    def retry(self, iid: str, delay_s: float = 0.0) -> bool:
        with self._mu:
            item = self._inflight.pop(iid, None)
            if item is None:
                return False
            self.stat["retried"] += 1
            self._delayed.append((time.monotonic() + delay_s, iid, item))
            return True

    def stats(self) -> Dict[str, int]:
        with self._mu:
            return dict(self.stat, ready=len(self._q), delayed=len(self._delayed), inflight=len(self._inflight))


class SqliteQueue:
    def __init__(self, path: str, name: str = "default", visibility_s: float = 60.0):
        self.name = name
        self.visibility_s = visibility_s
        self._mu = threading.Lock()
        self._db = sqlite3.connect(path, check_same_thread=False)
        self._db.execute("PRAGMA journal_mode=WAL")
        self._db.execute("CREATE TABLE IF NOT EXISTS q (id TEXT PRIMARY KEY, queue TEXT, body TEXT, state TEXT, "
                         "ready_at REAL, taken_at REAL, attempts INTEGER)")
        self._db.execute("CREATE INDEX IF NOT EXISTS q_ready ON q (queue, state, ready_at)")
        self._db.commit()

    def enqueue(self, item: Any, delay_s: float = 0.0) -> str:
        iid = uuid.uuid4().hex
        with self._mu:
            self._db.execute("INSERT INTO q VALUES (?, ?, ?, 'ready', ?, 0, 0)",
                             (iid, self.name, json.dumps(item), time.time() + delay_s))
            self._db.commit()
        return iid

    def reclaim_stale(self, now: Optional[float] = None) -> int:
        t = time.time() if now is None else now
        with self._mu:
            cur = self._db.execute("UPDATE q SET state='ready', ready_at=? WHERE queue=? AND state='inflight' "
                                   "AND taken_at < ?", (t, self.name, t - self.visibility_s))
            self._db.commit()
            return cur.rowcount

    def dequeue(self, now: Optional[float] = None) -> Optional[Tuple[str, Any]]:
        t = time.time() if now is None else now
        self.reclaim_stale(t)
        with self._mu:
            row = self._db.execute("SELECT id, body FROM q WHERE queue=? AND state='ready' AND ready_at <= ? "
                                   "ORDER BY ready_at LIMIT 1", (self.name, t)).fetchone()
            if row is None:
                return None
            self._db.execute("UPDATE q SET state='inflight', taken_at=?, attempts=attempts+1 WHERE id=?", (t, row[0]))
            self._db.commit()
            return row[0], json.loads(row[1])

    def ack(self, iid: str) -> bool:
        with self._mu:
            cur = self._db.execute("DELETE FROM q WHERE id=? AND state='inflight'", (iid,))
            self._db.commit()
            return cur.rowcount == 1

    def retry(self, iid: str, delay_s: float = 0.0) -> bool:
        with self._mu:
            cur = self._db.execute("UPDATE q SET state='ready', ready_at=? WHERE id=? AND state='inflight'",
                                   (time.time() + delay_s, iid))
            self._db.commit()
            return cur.rowcount == 1

    def stats(self) -> Dict[str, int]:
        with self._mu:
            rows = self._db.execute("SELECT state, COUNT(*) FROM q WHERE queue=? GROUP BY state", (self.name,)).fetchall()
        d = {"ready": 0, "inflight": 0}
        d.update({s: n for s, n in rows})
        return d
