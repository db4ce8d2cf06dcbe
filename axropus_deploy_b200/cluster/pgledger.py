"""The job ledger on PostgreSQL, over a Postgres frontend/backend protocol (v3) client
written here: no driver is needed.

:class:`PgConnection` opens one socket (``postgresql://user:password@host:port/db``),
authenticates with SCRAM-SHA-256 (RFC 5802 / RFC 7677, the server default since Postgres
14), MD5 or cleartext, and runs each statement through the extended query protocol
(Parse / Bind / Describe / Execute / Sync) with every parameter sent as text and typed by
the server, so values never enter the SQL text. Results come back as dicts; integer,
float and boolean columns are converted by their type OID.

:class:`PostgresLedger` is :class:`~.ledger.SqliteLedger` with its SQL carried over to
Postgres: ``?`` placeholders become ``$n``; ``INSERT OR REPLACE`` becomes ``INSERT ...
ON CONFLICT (primary key) DO UPDATE``; ``REAL`` columns become ``DOUBLE PRECISION`` and
``INTEGER`` columns ``BIGINT``; every table gets a trailing ``rowid BIGSERIAL`` column, which
gives the insertion order the SQLite ledger reads from its implicit rowid (it is left out
of ``SELECT *`` results). Same tables, columns and methods; :func:`build_ledger` picks it
with ``KORITH_LEDGER_BACKEND=postgres`` and ``KORITH_LEDGER_DSN``.

Reference: platform/ledger/postgres_store.py (the Postgres store), platform/ledger/store.py:10-52
(the protocol) and platform/runtime/config.py:118-124 (selection).
"""
from __future__ import annotations

import base64
import hashlib
import hmac
import os
import re
import socket
import struct
import threading
import urllib.parse
from typing import Any, Dict, List, Optional, Sequence, Tuple

from .ledger import _SCHEMA, SqliteLedger


class PgError(RuntimeError):
    def __init__(self, fields: Dict[str, str]):
        self.fields = fields
        self.code = fields.get("C", "")
        super().__init__(f"{fields.get('S', 'ERROR')} {self.code}: {fields.get('M', '')}")


_INT_OIDS = {20, 21, 23, 26}
_FLOAT_OIDS = {700, 701, 1700}
_BOOL_OID = 16


class _Result:
    def __init__(self, rows: List[Dict[str, Any]], rowcount: int):
        self.rows, self.rowcount = rows, rowcount


class PgConnection:
    def __init__(self, dsn: str, timeout_s: float = 30.0):
        u = urllib.parse.urlsplit(dsn)
        q = dict(urllib.parse.parse_qsl(u.query))
        self.user = urllib.parse.unquote(u.username or q.get("user") or os.environ.get("PGUSER", "postgres"))
        self.password = urllib.parse.unquote(u.password or q.get("password") or os.environ.get("PGPASSWORD", ""))
        self.database = (u.path or "/").lstrip("/") or q.get("dbname") or self.user
        self._sock = socket.create_connection((u.hostname or "127.0.0.1", u.port or 5432), timeout=timeout_s)
        self._buf = b""
        self._mu = threading.Lock()
        self.params: Dict[str, str] = {}
        self._startup()

    # ------------------------------------------------------------------ framing
    def _send(self, kind: bytes, payload: bytes = b"") -> None:
        self._sock.sendall(kind + struct.pack("!I", len(payload) + 4) + payload)

    def _recv(self) -> Tuple[bytes, bytes]:
        while len(self._buf) < 5:
            self._more()
        kind, n = self._buf[:1], struct.unpack("!I", self._buf[1:5])[0]
        while len(self._buf) < 1 + n:
            self._more()
        body, self._buf = self._buf[5:1 + n], self._buf[1 + n:]
        return kind, body

    def _more(self) -> None:
        chunk = self._sock.recv(65536)
        if not chunk:
            raise ConnectionError("postgres connection closed")
        self._buf += chunk

    @staticmethod
    def _cstr(s: str) -> bytes:
        return s.encode("utf-8") + b"\0"

    @staticmethod
    def _fields(body: bytes) -> Dict[str, str]:
        out = {}
        for part in body.split(b"\0"):
            if part:
                out[chr(part[0])] = part[1:].decode("utf-8", "replace")
        return out

    # ------------------------------------------------------------------ start-up and authentication
    def _startup(self) -> None:
        body = struct.pack("!I", 196608) + self._cstr("user") + self._cstr(self.user) + \
            self._cstr("database") + self._cstr(self.database) + self._cstr("client_encoding") + self._cstr("UTF8") + b"\0"
        self._sock.sendall(struct.pack("!I", len(body) + 4) + body)
        scram = None
        while True:
            kind, body = self._recv()
            if kind == b"R":
                code = struct.unpack("!I", body[:4])[0]
                if code == 0:
                    continue
                if code == 3:
                    self._send(b"p", self._cstr(self.password))
                elif code == 5:
                    inner = hashlib.md5((self.password + self.user).encode()).hexdigest()
                    self._send(b"p", self._cstr("md5" + hashlib.md5(inner.encode() + body[4:8]).hexdigest()))
                elif code == 10:
                    mechs = [m.decode() for m in body[4:].split(b"\0") if m]
                    if "SCRAM-SHA-256" not in mechs:
                        raise PgError({"M": f"no supported SASL mechanism in {mechs}"})
                    scram = _Scram(self.password)
                    first = scram.client_first().encode()
                    self._send(b"p", self._cstr("SCRAM-SHA-256") + struct.pack("!i", len(first)) + first)
                elif code == 11:
                    self._send(b"p", scram.client_final(body[4:].decode()).encode())
                elif code == 12:
                    scram.verify_server(body[4:].decode())
                else:
                    raise PgError({"M": f"unsupported authentication request {code}"})
            elif kind == b"S":
                k, v = body.split(b"\0")[:2]
                self.params[k.decode()] = v.decode()
            elif kind == b"E":
                raise PgError(self._fields(body))
            elif kind == b"Z":
                return
            # K (backend key data) and N (notices) need no answer

    # ------------------------------------------------------------------ queries
    def execute(self, sql: str, params: Sequence[Any] = ()) -> _Result:
        with self._mu:
            vals = []
            for v in params:
                if v is None:
                    vals.append(struct.pack("!i", -1))
                else:
                    b = (("t" if v else "f") if isinstance(v, bool) else str(v)).encode("utf-8")
                    vals.append(struct.pack("!i", len(b)) + b)
            self._send(b"P", self._cstr("") + self._cstr(sql) + struct.pack("!H", 0))
            self._send(b"B", self._cstr("") + self._cstr("") + struct.pack("!H", 0) + struct.pack("!H", len(vals))
                       + b"".join(vals) + struct.pack("!H", 0))
            self._send(b"D", b"P" + self._cstr(""))
            self._send(b"E", self._cstr("") + struct.pack("!I", 0))
            self._send(b"S")
            cols: List[Tuple[str, int]] = []
            rows: List[Dict[str, Any]] = []
            count, err = 0, None
            while True:
                kind, body = self._recv()
                if kind == b"T":
                    n = struct.unpack("!H", body[:2])[0]
                    off, cols = 2, []
                    for _ in range(n):
                        end = body.index(b"\0", off)
                        name = body[off:end].decode()
                        oid = struct.unpack("!I", body[end + 7:end + 11])[0]
                        cols.append((name, oid))
                        off = end + 19
                elif kind == b"D":
                    n = struct.unpack("!H", body[:2])[0]
                    off, row = 2, {}
                    for i in range(n):
                        ln = struct.unpack("!i", body[off:off + 4])[0]
                        off += 4
                        if ln < 0:
                            row[cols[i][0]] = None
                            continue
                        row[cols[i][0]] = self._convert(body[off:off + ln].decode("utf-8"), cols[i][1])
                        off += ln
                    rows.append(row)
                elif kind == b"C":
                    tag = body.rstrip(b"\0").decode().split()
                    count = int(tag[-1]) if tag and tag[-1].isdigit() else 0
                elif kind == b"E":
                    err = PgError(self._fields(body))
                elif kind == b"Z":
                    if err is not None:
                        raise err
                    return _Result(rows, count)
                # '1' parse, '2' bind, 'n' no data, 'N' notice, 'S' parameter status: nothing to keep

    @staticmethod
    def _convert(text: str, oid: int) -> Any:
        if oid in _INT_OIDS:
            return int(text)
        if oid in _FLOAT_OIDS:
            return float(text)
        if oid == _BOOL_OID:
            return text == "t"
        return text

    def close(self) -> None:
        try:
            self._send(b"X")
        except OSError:
            pass
        self._sock.close()


class _Scram:
    """Client side of SCRAM-SHA-256 without channel binding (``n,,`` GS2 header)."""

    def __init__(self, password: str):
        self.password = password
        self.nonce = base64.b64encode(os.urandom(18)).decode()

    def client_first(self) -> str:
        self.first_bare = f"n=,r={self.nonce}"
        return "n,," + self.first_bare

    def client_final(self, server_first: str) -> str:
        a = dict(kv.split("=", 1) for kv in server_first.split(","))
        if not a["r"].startswith(self.nonce):
            raise PgError({"M": "SCRAM server nonce does not extend the client nonce"})
        salted = hashlib.pbkdf2_hmac("sha256", self.password.encode("utf-8"), base64.b64decode(a["s"]), int(a["i"]))
        client_key = hmac.new(salted, b"Client Key", hashlib.sha256).digest()
        stored = hashlib.sha256(client_key).digest()
        without_proof = f"c=biws,r={a['r']}"
        self.auth_message = f"{self.first_bare},{server_first},{without_proof}".encode()
        sig = hmac.new(stored, self.auth_message, hashlib.sha256).digest()
        proof = bytes(x ^ y for x, y in zip(client_key, sig))
        self.server_key = hmac.new(salted, b"Server Key", hashlib.sha256).digest()
        return f"{without_proof},p={base64.b64encode(proof).decode()}"

    def verify_server(self, server_final: str) -> None:
        want = hmac.new(self.server_key, self.auth_message, hashlib.sha256).digest()
        got = dict(kv.split("=", 1) for kv in server_final.split(",")).get("v", "")
        if not hmac.compare_digest(base64.b64decode(got), want):
            raise PgError({"M": "SCRAM server signature mismatch"})


# ---------------------------------------------------------------------- ledger
def _pg_schema(stmt: str) -> str:
    s = re.sub(r"\bREAL\b", "DOUBLE PRECISION", stmt)
    s = re.sub(r"\bINTEGER\b", "BIGINT", s)
    if s.lstrip().upper().startswith("CREATE TABLE"):
        i = s.rindex(")")
        s = s[:i] + ", rowid BIGSERIAL" + s[i:]
    return s


def _table_keys() -> Dict[str, Tuple[List[str], List[str]]]:
    """table -> (columns in order, primary key columns), read from the shared schema."""
    out = {}
    for stmt in _SCHEMA:
        m = re.match(r"\s*CREATE TABLE IF NOT EXISTS (\w+) \((.*)\)\s*$", stmt, re.S)
        if not m:
            continue
        body = m.group(2)
        pk = re.search(r"PRIMARY KEY \(([^)]*)\)", body)
        cols, keys = [], []
        for part in re.split(r",(?![^()]*\))", body):
            part = part.strip()
            if not part or part.upper().startswith("PRIMARY KEY"):
                continue
            name = part.split()[0]
            cols.append(name)
            if "PRIMARY KEY" in part.upper():
                keys.append(name)
        if pk:
            keys = [k.strip() for k in pk.group(1).split(",")]
        out[m.group(1)] = (cols, keys)
    return out


_TABLES = _table_keys()


def translate(sql: str) -> str:
    """SQLite ledger SQL -> Postgres."""
    m = re.match(r"\s*INSERT OR REPLACE INTO (\w+) (.*)$", sql, re.S)
    if m:
        cols, keys = _TABLES[m.group(1)]
        upd = ", ".join(f"{c}=EXCLUDED.{c}" for c in cols if c not in keys)
        sql = f"INSERT INTO {m.group(1)} {m.group(2)} ON CONFLICT ({', '.join(keys)}) DO UPDATE SET {upd}"
    n = 0

    def num(_):
        nonlocal n
        n += 1
        return f"${n}"

    return re.sub(r"\?", num, sql)


class PostgresLedger(SqliteLedger):
    def __init__(self, dsn: str):
        if not dsn:
            raise ValueError("Postgres ledger needs a DSN (KORITH_LEDGER_DSN)")
        self.path = dsn
        self._mu = threading.Lock()
        self._pg = PgConnection(dsn)
        self.init()

    def init(self) -> None:
        for s in _SCHEMA:
            self._pg.execute(_pg_schema(s))

    def _exec(self, sql: str, args: tuple = ()) -> _Result:
        with self._mu:
            return self._pg.execute(translate(sql), args)

    def _rows(self, sql: str, args: tuple = ()) -> List[Dict[str, Any]]:
        with self._mu:
            rows = self._pg.execute(translate(sql), args).rows
        if re.search(r"SELECT\s+\*", sql):
            for r in rows:
                r.pop("rowid", None)
        return rows

    def close(self) -> None:
        self._pg.close()


def build_ledger(path: Optional[str] = None):
    """``KORITH_LEDGER_BACKEND=postgres`` with ``KORITH_LEDGER_DSN``, else the SQLite file
    ``path`` (default ``KORITH_PLATFORM_DB``)."""
    if os.environ.get("KORITH_LEDGER_BACKEND", "sqlite").strip().lower() == "postgres":
        return PostgresLedger(os.environ.get("KORITH_LEDGER_DSN", ""))
    p = path or os.environ.get("KORITH_PLATFORM_DB", "./platform_data/ledger.sqlite")
    if p != ":memory:":
        os.makedirs(os.path.dirname(os.path.abspath(p)), exist_ok=True)
    return SqliteLedger(p)
