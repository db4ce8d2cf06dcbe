"""Job ledger of the control plane: jobs, runs, KV snapshots, API keys, replay and
speculative-decoding governance, and where each snapshot lives.

One SQLite file (WAL, one connection per thread). The tables and their columns carry
the reference's names so that an existing ledger database opens unchanged and tools
that query it keep working; every job row also stores an ``immutable_hash`` (sha256 of
its canonical jobspec JSON), which :meth:`SqliteLedger.verify_job` re-checks.

Reference: platform/ledger/store.py:10-52 (the ``LedgerStore`` protocol) and
platform/ledger/db.py:30-147 (table layout).
"""
from __future__ import annotations

import hashlib
import json
import sqlite3
import threading
from typing import Any, Dict, List, Optional

_SCHEMA = [
    """CREATE TABLE IF NOT EXISTS jobs (job_id TEXT PRIMARY KEY, created_at TEXT NOT NULL,
       org_id TEXT NOT NULL DEFAULT 'default', jobspec_json TEXT NOT NULL, fingerprint_json TEXT NOT NULL,
       prompt_hash TEXT NOT NULL, fingerprint_hash TEXT NOT NULL, idempotency_key TEXT, status TEXT NOT NULL,
       immutable_hash TEXT NOT NULL)""",
    "CREATE INDEX IF NOT EXISTS idx_jobs_fp ON jobs(fingerprint_hash, org_id)",
    "CREATE INDEX IF NOT EXISTS idx_jobs_idem ON jobs(idempotency_key, org_id)",
    """CREATE TABLE IF NOT EXISTS runs (run_id TEXT PRIMARY KEY, job_id TEXT NOT NULL,
       org_id TEXT NOT NULL DEFAULT 'default', started_at TEXT NOT NULL, finished_at TEXT NOT NULL,
       exit_code INTEGER NOT NULL, metrics_path TEXT NOT NULL, events_path TEXT NOT NULL,
       output_path TEXT NOT NULL, log_path TEXT NOT NULL)""",
    "CREATE INDEX IF NOT EXISTS idx_runs_job ON runs(job_id)",
    """CREATE TABLE IF NOT EXISTS snapshots (snapshot_id TEXT PRIMARY KEY, job_id TEXT NOT NULL,
       org_id TEXT NOT NULL DEFAULT 'default', fingerprint_hash TEXT NOT NULL, snapshot_path TEXT NOT NULL,
       created_at TEXT NOT NULL)""",
    "CREATE INDEX IF NOT EXISTS idx_snapshots_job_id ON snapshots(job_id)",
    """CREATE TABLE IF NOT EXISTS api_keys (key_id TEXT PRIMARY KEY, key_hash TEXT NOT NULL UNIQUE,
       org_id TEXT NOT NULL, created_at TEXT NOT NULL, revoked_at TEXT,
       rate_limit_tpm INTEGER NOT NULL DEFAULT 120000, rate_limit_rpm INTEGER NOT NULL DEFAULT 600,
       permissions_json TEXT NOT NULL DEFAULT '{}')""",
    """CREATE TABLE IF NOT EXISTS replay_governance (fingerprint_hash TEXT PRIMARY KEY,
       replay_disabled INTEGER NOT NULL DEFAULT 0, disabled_reason TEXT, disabled_at TEXT,
       cooldown_until REAL NOT NULL DEFAULT 0, negative_roi_streak INTEGER NOT NULL DEFAULT 0,
       corruption_detected INTEGER NOT NULL DEFAULT 0, restore_guard_disabled INTEGER NOT NULL DEFAULT 0,
       updated_at TEXT NOT NULL)""",
    """CREATE TABLE IF NOT EXISTS spec_governance (fingerprint_hash TEXT PRIMARY KEY,
       org_id TEXT NOT NULL DEFAULT 'default', spec_disabled INTEGER NOT NULL DEFAULT 0, reason TEXT,
       cooldown_until REAL NOT NULL DEFAULT 0, bad_accept_streak INTEGER NOT NULL DEFAULT 0,
       updated_at TEXT NOT NULL)""",
    """CREATE TABLE IF NOT EXISTS snapshot_locations (fingerprint_hash TEXT NOT NULL, snapshot_id TEXT NOT NULL,
       org_id TEXT NOT NULL, node_id TEXT NOT NULL, worker_id TEXT, snapshot_path TEXT NOT NULL,
       size_bytes INTEGER NOT NULL DEFAULT 0, created_at TEXT NOT NULL, last_used_at TEXT NOT NULL,
       PRIMARY KEY (fingerprint_hash, org_id, node_id, snapshot_id))""",
]


def canonical_json(obj: Any) -> str:
    return json.dumps(obj, sort_keys=True, separators=(",", ":"), ensure_ascii=False)


def sha256_hex(s: str) -> str:
    return hashlib.sha256(s.encode("utf-8")).hexdigest()


class SqliteLedger:
    """The ledger on one SQLite file (``":memory:"`` keeps it in this process)."""

    def __init__(self, path: str = ":memory:"):
        self.path = path
        self._local = threading.local()
        self._mu = threading.Lock()
        self._shared = sqlite3.connect(path, check_same_thread=False) if path == ":memory:" else None
        self.init()

    # ------------------------------------------------------------------ plumbing
    def _conn(self) -> sqlite3.Connection:
        if self._shared is not None:
            return self._shared
        c = getattr(self._local, "conn", None)
        if c is None:
            c = sqlite3.connect(self.path, timeout=10.0)
            c.execute("PRAGMA journal_mode=WAL")
            self._local.conn = c
        return c

    def _exec(self, sql: str, args: tuple = ()) -> sqlite3.Cursor:
        with self._mu:
            c = self._conn()
            cur = c.execute(sql, args)
            c.commit()
            return cur

    def _rows(self, sql: str, args: tuple = ()) -> List[Dict[str, Any]]:
        with self._mu:
            cur = self._conn().execute(sql, args)
            cols = [d[0] for d in cur.description]
            return [dict(zip(cols, r)) for r in cur.fetchall()]

    def _row(self, sql: str, args: tuple = ()) -> Optional[Dict[str, Any]]:
        rows = self._rows(sql, args)
        return rows[0] if rows else None

    def init(self) -> None:
        for s in _SCHEMA:
            self._exec(s)

    # ------------------------------------------------------------------ jobs and runs
    def insert_job(self, job_id: str, created_at: str, jobspec: Dict[str, Any], fingerprint: Dict[str, Any],
                   prompt_hash: str, fingerprint_hash: str, idempotency_key: Optional[str], status: str,
                   org_id: str = "default") -> None:
        spec = canonical_json(jobspec)
        self._exec("INSERT INTO jobs VALUES (?,?,?,?,?,?,?,?,?,?)",
                   (job_id, created_at, org_id, spec, canonical_json(fingerprint), prompt_hash, fingerprint_hash,
                    idempotency_key, status, sha256_hex(spec)))

    def update_status(self, job_id: str, new_status: str) -> None:
        self._exec("UPDATE jobs SET status=? WHERE job_id=?", (new_status, job_id))

    def get_job(self, job_id: str) -> Optional[Dict[str, Any]]:
        return self._row("SELECT * FROM jobs WHERE job_id=?", (job_id,))

    def verify_job(self, job_id: str) -> bool:
        """The stored jobspec still hashes to the value recorded at insert time."""
        j = self.get_job(job_id)
        return j is not None and sha256_hex(j["jobspec_json"]) == j["immutable_hash"]

    def list_jobs(self, limit: int, org_id: Optional[str] = None) -> List[Dict[str, Any]]:
        if org_id is None:
            return self._rows("SELECT * FROM jobs ORDER BY created_at DESC, rowid DESC LIMIT ?", (int(limit),))
        return self._rows("SELECT * FROM jobs WHERE org_id=? ORDER BY created_at DESC, rowid DESC LIMIT ?",
                          (org_id, int(limit)))

    def find_job_by_fingerprint(self, fingerprint_hash: str, org_id: Optional[str] = None) -> Optional[str]:
        q = "SELECT job_id FROM jobs WHERE fingerprint_hash=?" + (" AND org_id=?" if org_id else "")
        r = self._row(q + " ORDER BY created_at DESC LIMIT 1", (fingerprint_hash, org_id) if org_id else
                      (fingerprint_hash,))
        return r["job_id"] if r else None

    def find_job_by_idempotency(self, idempotency_key: str, org_id: Optional[str] = None) -> Optional[str]:
        q = "SELECT job_id FROM jobs WHERE idempotency_key=?" + (" AND org_id=?" if org_id else "")
        r = self._row(q + " LIMIT 1", (idempotency_key, org_id) if org_id else (idempotency_key,))
        return r["job_id"] if r else None

    def insert_run(self, run_id: str, job_id: str, started_at: str, finished_at: str, exit_code: int,
                   metrics_path: str, events_path: str, output_path: str, log_path: str,
                   org_id: str = "default") -> None:
        self._exec("INSERT INTO runs VALUES (?,?,?,?,?,?,?,?,?,?)",
                   (run_id, job_id, org_id, started_at, finished_at, int(exit_code), metrics_path, events_path,
                    output_path, log_path))

    def get_latest_run(self, job_id: str) -> Optional[Dict[str, Any]]:
        return self._row("SELECT * FROM runs WHERE job_id=? ORDER BY finished_at DESC, rowid DESC LIMIT 1",
                         (job_id,))

    # ------------------------------------------------------------------ snapshots
    def insert_snapshot(self, snapshot_id: str, job_id: str, fingerprint_hash: str, snapshot_path: str,
                        created_at: str, org_id: str = "default") -> None:
        self._exec("INSERT OR REPLACE INTO snapshots VALUES (?,?,?,?,?,?)",
                   (snapshot_id, job_id, org_id, fingerprint_hash, snapshot_path, created_at))

    def get_snapshot_for_job(self, job_id: str) -> Optional[Dict[str, Any]]:
        return self._row("SELECT * FROM snapshots WHERE job_id=? ORDER BY created_at DESC LIMIT 1", (job_id,))

    def upsert_snapshot_location(self, fingerprint_hash: str, snapshot_id: str, org_id: str, node_id: str,
                                 worker_id: Optional[str], snapshot_path: str, size_bytes: int,
                                 created_at: str, last_used_at: str) -> None:
        self._exec("INSERT INTO snapshot_locations VALUES (?,?,?,?,?,?,?,?,?) ON CONFLICT"
                   "(fingerprint_hash, org_id, node_id, snapshot_id) DO UPDATE SET worker_id=excluded.worker_id, "
                   "snapshot_path=excluded.snapshot_path, size_bytes=excluded.size_bytes, "
                   "last_used_at=excluded.last_used_at",
                   (fingerprint_hash, snapshot_id, org_id, node_id, worker_id, snapshot_path, int(size_bytes),
                    created_at, last_used_at))

    def list_snapshot_locations(self, fingerprint_hash: str, org_id: str) -> List[Dict[str, Any]]:
        return self._rows("SELECT * FROM snapshot_locations WHERE fingerprint_hash=? AND org_id=? "
                          "ORDER BY last_used_at DESC", (fingerprint_hash, org_id))

    def mark_snapshot_location_used(self, fingerprint_hash: str, org_id: str, node_id: str, snapshot_id: str,
                                    last_used_at: str) -> None:
        self._exec("UPDATE snapshot_locations SET last_used_at=? WHERE fingerprint_hash=? AND org_id=? AND "
                   "node_id=? AND snapshot_id=?", (last_used_at, fingerprint_hash, org_id, node_id, snapshot_id))

    def prune_snapshot_locations(self, max_entries_per_fingerprint: int = 8) -> int:
        """Keep the most recently used ``max_entries_per_fingerprint`` locations of each
        (fingerprint, org); returns the number removed."""
        rows = self._rows("SELECT rowid, fingerprint_hash, org_id FROM snapshot_locations "
                          "ORDER BY fingerprint_hash, org_id, last_used_at DESC")
        seen: Dict[tuple, int] = {}
        drop = []
        for r in rows:
            k = (r["fingerprint_hash"], r["org_id"])
            seen[k] = seen.get(k, 0) + 1
            if seen[k] > max_entries_per_fingerprint:
                drop.append(r["rowid"])
        for rid in drop:
            self._exec("DELETE FROM snapshot_locations WHERE rowid=?", (rid,))
        return len(drop)

    # ------------------------------------------------------------------ API keys
    def create_api_key(self, key_id: str, key_hash: str, org_id: str, created_at: str, rate_limit_tpm: int,
                       rate_limit_rpm: int, permissions_json: str) -> None:
        self._exec("INSERT INTO api_keys VALUES (?,?,?,?,NULL,?,?,?)",
                   (key_id, key_hash, org_id, created_at, int(rate_limit_tpm), int(rate_limit_rpm), permissions_json))

    def revoke_api_key(self, key_id: str, revoked_at: str) -> bool:
        return self._exec("UPDATE api_keys SET revoked_at=? WHERE key_id=? AND revoked_at IS NULL",
                          (revoked_at, key_id)).rowcount == 1

    def list_api_keys(self, org_id: Optional[str] = None) -> List[Dict[str, Any]]:
        cols = "key_id, org_id, created_at, revoked_at, rate_limit_tpm, rate_limit_rpm, permissions_json"
        if org_id is None:
            return self._rows(f"SELECT {cols} FROM api_keys ORDER BY created_at")
        return self._rows(f"SELECT {cols} FROM api_keys WHERE org_id=? ORDER BY created_at", (org_id,))

    def get_api_key_by_hash(self, key_hash: str) -> Optional[Dict[str, Any]]:
        return self._row("SELECT * FROM api_keys WHERE key_hash=?", (key_hash,))

    # ------------------------------------------------------------------ governance
    def upsert_replay_governance(self, fingerprint_hash: str, replay_disabled: int, disabled_reason: Optional[str],
                                 disabled_at: Optional[str], cooldown_until: float, negative_roi_streak: int,
                                 corruption_detected: int, restore_guard_disabled: int, updated_at: str) -> None:
        self._exec("INSERT OR REPLACE INTO replay_governance VALUES (?,?,?,?,?,?,?,?,?)",
                   (fingerprint_hash, int(replay_disabled), disabled_reason, disabled_at, float(cooldown_until),
                    int(negative_roi_streak), int(corruption_detected), int(restore_guard_disabled), updated_at))

    def get_replay_governance(self, fingerprint_hash: str) -> Optional[Dict[str, Any]]:
        return self._row("SELECT * FROM replay_governance WHERE fingerprint_hash=?", (fingerprint_hash,))

    def list_replay_governance(self, limit: int = 100) -> List[Dict[str, Any]]:
        return self._rows("SELECT * FROM replay_governance ORDER BY updated_at DESC LIMIT ?", (int(limit),))

    def upsert_spec_governance(self, fingerprint_hash: str, org_id: str, spec_disabled: int, reason: Optional[str],
                               cooldown_until: float, bad_accept_streak: int, updated_at: str) -> None:
        self._exec("INSERT OR REPLACE INTO spec_governance VALUES (?,?,?,?,?,?,?)",
                   (fingerprint_hash, org_id, int(spec_disabled), reason, float(cooldown_until),
                    int(bad_accept_streak), updated_at))

    def get_spec_governance(self, fingerprint_hash: str) -> Optional[Dict[str, Any]]:
        return self._row("SELECT * FROM spec_governance WHERE fingerprint_hash=?", (fingerprint_hash,))

    def list_spec_governance(self, limit: int = 100, org_id: Optional[str] = None) -> List[Dict[str, Any]]:
        if org_id is None:
            return self._rows("SELECT * FROM spec_governance ORDER BY updated_at DESC LIMIT ?", (int(limit),))
        return self._rows("SELECT * FROM spec_governance WHERE org_id=? ORDER BY updated_at DESC LIMIT ?",
                          (org_id, int(limit)))
