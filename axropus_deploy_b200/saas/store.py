"""SQLite store of the hosted backend: customers, API keys, deployments, usage metrics and
invoices, plus the password hashing and the signed access tokens of its accounts.

The tables keep the reference backend's column names (backend/models.py:9-111) so usage data
exported from one reads in the other; the storage here is plain ``sqlite3`` behind one lock
(one backend process, WAL journal) instead of an ORM. Access tokens are JSON Web Tokens
(RFC 7519) signed with HMAC-SHA256 (``alg`` HS256), written with ``hmac`` / ``base64``.
"""
from __future__ import annotations

import base64
import hashlib
import hmac
import json
import secrets
import sqlite3
import threading
import time
from datetime import datetime, timedelta, timezone
from typing import Any, Dict, List, Optional

import bcrypt

SCHEMA = """
CREATE TABLE IF NOT EXISTS customers (
  id INTEGER PRIMARY KEY AUTOINCREMENT, email TEXT UNIQUE NOT NULL, password_hash TEXT NOT NULL,
  company_name TEXT, created_at TEXT NOT NULL);
CREATE TABLE IF NOT EXISTS api_keys (
  id INTEGER PRIMARY KEY AUTOINCREMENT, customer_id INTEGER NOT NULL REFERENCES customers(id) ON DELETE CASCADE,
  key TEXT UNIQUE NOT NULL, status TEXT NOT NULL DEFAULT 'trial', tier TEXT NOT NULL DEFAULT 'trial',
  created_at TEXT NOT NULL, expires_at TEXT);
CREATE TABLE IF NOT EXISTS deployments (
  id INTEGER PRIMARY KEY AUTOINCREMENT, customer_id INTEGER NOT NULL REFERENCES customers(id) ON DELETE CASCADE,
  api_key_id INTEGER REFERENCES api_keys(id), runtime TEXT NOT NULL, model_family TEXT NOT NULL,
  model_size TEXT NOT NULL, draft_model TEXT, inference_url TEXT, status TEXT NOT NULL DEFAULT 'pending',
  deployed_at TEXT);
CREATE TABLE IF NOT EXISTS metrics (
  id INTEGER PRIMARY KEY AUTOINCREMENT, api_key_id INTEGER NOT NULL REFERENCES api_keys(id) ON DELETE CASCADE,
  timestamp TEXT NOT NULL, tokens_processed INTEGER NOT NULL DEFAULT 0, interval_seconds INTEGER NOT NULL DEFAULT 60,
  prefix_skipped INTEGER NOT NULL DEFAULT 0, decode_accelerated INTEGER NOT NULL DEFAULT 0,
  amf_hit_rate REAL NOT NULL DEFAULT 0, spec_acceptance_rate REAL NOT NULL DEFAULT 0,
  effective_tps REAL NOT NULL DEFAULT 0, baseline_tps REAL NOT NULL DEFAULT 0, compute_saved_pct REAL NOT NULL DEFAULT 0,
  gpu_count INTEGER NOT NULL DEFAULT 0, model_family TEXT, model_size_bucket TEXT, adapter_type TEXT,
  sdk_version TEXT, license_id TEXT, heartbeat INTEGER NOT NULL DEFAULT 0);
CREATE INDEX IF NOT EXISTS metrics_key_ts ON metrics(api_key_id, timestamp);
CREATE TABLE IF NOT EXISTS invoices (
  id INTEGER PRIMARY KEY AUTOINCREMENT, customer_id INTEGER NOT NULL REFERENCES customers(id) ON DELETE CASCADE,
  period_start TEXT, period_end TEXT, total_tokens INTEGER, amount_cents INTEGER,
  status TEXT NOT NULL DEFAULT 'pending', created_at TEXT NOT NULL);
"""

TIERS = ("trial", "standard", "enterprise")
TRIAL_DAYS = 14


def utcnow() -> datetime:
    return datetime.now(timezone.utc).replace(tzinfo=None, microsecond=0)


def iso(t: Optional[datetime]) -> Optional[str]:
    return None if t is None else t.isoformat(sep=" ")


def parse_ts(s: Optional[str]) -> Optional[datetime]:
    if s is None:
        return None
    t = datetime.fromisoformat(str(s).replace("Z", "+00:00"))
    return t.astimezone(timezone.utc).replace(tzinfo=None) if t.tzinfo else t


def new_key_value() -> str:
    """API keys are ``ax-`` + 32 hex digits (the prefix clients and workers check)."""
    return "ax-" + secrets.token_hex(16)


def hash_password(password: str) -> str:
    return bcrypt.hashpw(password.encode(), bcrypt.gensalt(rounds=10)).decode()


def verify_password(password: str, password_hash: str) -> bool:
    try:
        return bcrypt.checkpw(password.encode(), password_hash.encode())
    except ValueError:
        return False


def _b64(b: bytes) -> str:
    return base64.urlsafe_b64encode(b).rstrip(b"=").decode()


def _unb64(s: str) -> bytes:
    return base64.urlsafe_b64decode(s + "=" * (-len(s) % 4))


def make_token(secret: str, customer_id: int, ttl_s: int = 86400, now: Optional[float] = None) -> str:
    now = time.time() if now is None else now
    head = _b64(json.dumps({"alg": "HS256", "typ": "JWT"}, separators=(",", ":")).encode())
    body = _b64(json.dumps({"sub": str(customer_id), "iat": int(now), "exp": int(now + ttl_s)},
                           separators=(",", ":")).encode())
    sig = hmac.new(secret.encode(), f"{head}.{body}".encode(), hashlib.sha256).digest()
    return f"{head}.{body}.{_b64(sig)}"


def read_token(secret: str, token: str, now: Optional[float] = None) -> int:
    """Customer id of a valid, unexpired token; ValueError otherwise."""
    try:
        head, body, sig = token.split(".")
        want = hmac.new(secret.encode(), f"{head}.{body}".encode(), hashlib.sha256).digest()
        if not hmac.compare_digest(want, _unb64(sig)):
            raise ValueError("bad signature")
        if json.loads(_unb64(head)).get("alg") != "HS256":
            raise ValueError("bad algorithm")
        claims = json.loads(_unb64(body))
    except ValueError:
        raise
    except Exception as e:
        raise ValueError(f"malformed token: {e}") from None
    if claims.get("exp", 0) < (time.time() if now is None else now):
        raise ValueError("expired")
    return int(claims["sub"])


class Store:
    def __init__(self, path: str = ":memory:"):
        self.db = sqlite3.connect(path, check_same_thread=False)
        self.db.row_factory = sqlite3.Row
        self.mu = threading.Lock()
        with self.mu:
            self.db.execute("PRAGMA foreign_keys = ON")
            if path != ":memory:":
                self.db.execute("PRAGMA journal_mode = WAL")
            self.db.executescript(SCHEMA)
            self.db.commit()

    def q(self, sql: str, args=()) -> List[Dict[str, Any]]:
        with self.mu:
            return [dict(r) for r in self.db.execute(sql, args).fetchall()]

    def one(self, sql: str, args=()) -> Optional[Dict[str, Any]]:
        rows = self.q(sql, args)
        return rows[0] if rows else None

    def exec(self, sql: str, args=()) -> int:
        with self.mu:
            cur = self.db.execute(sql, args)
            self.db.commit()
            return int(cur.lastrowid or 0)

    def ping(self) -> bool:
        try:
            self.q("SELECT 1")
            return True
        except sqlite3.Error:
            return False

    # accounts and keys
    def add_customer(self, email: str, password: str, company: Optional[str]) -> int:
        return self.exec("INSERT INTO customers (email, password_hash, company_name, created_at) VALUES (?,?,?,?)",
                         (email.lower(), hash_password(password), company, iso(utcnow())))

    def add_key(self, customer_id: int, tier: str = "trial") -> Dict[str, Any]:
        if tier not in TIERS:
            raise ValueError(f"tier must be one of {TIERS}")
        now = utcnow()
        exp = now + timedelta(days=TRIAL_DAYS) if tier == "trial" else None
        value = new_key_value()
        kid = self.exec("INSERT INTO api_keys (customer_id, key, status, tier, created_at, expires_at) "
                        "VALUES (?,?,?,?,?,?)",
                        (customer_id, value, "trial" if tier == "trial" else "active", tier, iso(now), iso(exp)))
        return self.one("SELECT * FROM api_keys WHERE id=?", (kid,))

    def active_key(self, value: str) -> Optional[Dict[str, Any]]:
        """The key row when it exists, is not revoked and has not expired."""
        if not isinstance(value, str) or not value.startswith("ax-"):
            return None
        row = self.one("SELECT * FROM api_keys WHERE key=?", (value,))
        if row is None or row["status"] == "revoked":
            return None
        exp = parse_ts(row["expires_at"])
        if exp is not None and exp <= utcnow():
            return None
        return row
