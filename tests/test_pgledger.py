"""The Postgres ledger against an in-process fake server that speaks the Postgres v3
protocol (start-up, SCRAM-SHA-256 or MD5 authentication, extended query messages) and runs
the statements on SQLite. Every ledger method gives the same rows through Postgres as the
SQLite ledger does; a wrong password is refused.

Reference: platform/ledger/postgres_store.py and platform/tests (ledger round trips).
"""
import base64
import hashlib
import hmac
import os
import re
import socketserver
import sqlite3
import struct
import threading

import pytest

from axropus_deploy_b200.cluster.ledger import SqliteLedger
from axropus_deploy_b200.cluster.pgledger import PgError, PostgresLedger, build_ledger, translate


class _FakePg:
    def __init__(self, password="s3cret", auth="scram"):
        self.password, self.auth = password, auth
        self.db = sqlite3.connect(":memory:", check_same_thread=False)
        self.mu = threading.Lock()
        self.statements = []

    @staticmethod
    def to_sqlite(sql):
        s = sql.replace(", rowid BIGSERIAL", "").replace("DOUBLE PRECISION", "REAL")
        return re.sub(r"\$(\d+)", r":p\1", s)

    def run(self, sql, params):
        def val(b):
            if b is None:
                return None
            t = b.decode()
            if re.fullmatch(r"-?\d+", t):
                return int(t)
            if re.fullmatch(r"-?\d+\.\d*(e-?\d+)?", t):
                return float(t)
            return t
        with self.mu:
            self.statements.append(sql)
            cur = self.db.execute(self.to_sqlite(sql), {f"p{i + 1}": val(p) for i, p in enumerate(params)})
            rows = cur.fetchall()
            self.db.commit()
            return cur.description, rows, cur.rowcount

    def serve(self):
        fake = self

        class H(socketserver.BaseRequestHandler):
            def send(self, kind, body=b""):
                self.request.sendall(kind + struct.pack("!I", len(body) + 4) + body)

            def recv_exact(self, n):
                b = b""
                while len(b) < n:
                    c = self.request.recv(n - len(b))
                    if not c:
                        raise ConnectionError
                    b += c
                return b

            def msg(self):
                kind = self.recv_exact(1)
                n = struct.unpack("!I", self.recv_exact(4))[0]
                return kind, self.recv_exact(n - 4)

            def error(self, code, text):
                self.send(b"E", b"SERROR\0C" + code.encode() + b"\0M" + text.encode() + b"\0\0")

            def auth(self, user):
                if fake.auth == "md5":
                    salt = os.urandom(4)
                    self.send(b"R", struct.pack("!I", 5) + salt)
                    _, body = self.msg()
                    inner = hashlib.md5((fake.password + user).encode()).hexdigest()
                    want = "md5" + hashlib.md5(inner.encode() + salt).hexdigest()
                    return body.rstrip(b"\0").decode() == want
                self.send(b"R", struct.pack("!I", 10) + b"SCRAM-SHA-256\0\0")
                _, body = self.msg()
                mech_end = body.index(b"\0")
                first = body[mech_end + 5:].decode()
                first_bare = first[3:]
                cnonce = dict(kv.split("=", 1) for kv in first_bare.split(","))["r"]
                salt, iters = os.urandom(16), 4096
                nonce = cnonce + base64.b64encode(os.urandom(12)).decode()
                server_first = f"r={nonce},s={base64.b64encode(salt).decode()},i={iters}"
                self.send(b"R", struct.pack("!I", 11) + server_first.encode())
                _, body = self.msg()
                final = body.decode()
                without_proof, proof = final.rsplit(",p=", 1)
                salted = hashlib.pbkdf2_hmac("sha256", fake.password.encode(), salt, iters)
                ck = hmac.new(salted, b"Client Key", hashlib.sha256).digest()
                stored = hashlib.sha256(ck).digest()
                am = f"{first_bare},{server_first},{without_proof}".encode()
                sig = hmac.new(stored, am, hashlib.sha256).digest()
                got_ck = bytes(x ^ y for x, y in zip(base64.b64decode(proof), sig))
                if hashlib.sha256(got_ck).digest() != stored:
                    return False
                sk = hmac.new(salted, b"Server Key", hashlib.sha256).digest()
                self.send(b"R", struct.pack("!I", 12) + b"v=" + base64.b64encode(hmac.new(sk, am, hashlib.sha256)
                                                                                  .digest()))
                return True

            def handle(self):
                n = struct.unpack("!I", self.recv_exact(4))[0]
                body = self.recv_exact(n - 4)[4:]
                kv = body.split(b"\0")
                opts = {kv[i].decode(): kv[i + 1].decode() for i in range(0, len(kv) - 1, 2) if kv[i]}
                if not self.auth(opts["user"]):
                    self.error("28P01", f'password authentication failed for user "{opts["user"]}"')
                    return
                self.send(b"R", struct.pack("!I", 0))
                self.send(b"S", b"server_version\x0016.0\0")
                self.send(b"K", struct.pack("!II", 1, 2))
                self.send(b"Z", b"I")
                sql, params = None, []
                while True:
                    try:
                        kind, body = self.msg()
                    except ConnectionError:
                        return
                    if kind == b"X":
                        return
                    if kind == b"P":
                        parts = body.split(b"\0")
                        sql = parts[1].decode()
                    elif kind == b"B":
                        off = body.index(b"\0") + 1
                        off = body.index(b"\0", off) + 1
                        nf = struct.unpack("!H", body[off:off + 2])[0]
                        off += 2 + 2 * nf
                        npar = struct.unpack("!H", body[off:off + 2])[0]
                        off += 2
                        params = []
                        for _ in range(npar):
                            ln = struct.unpack("!i", body[off:off + 4])[0]
                            off += 4
                            params.append(None if ln < 0 else body[off:off + ln])
                            off += max(ln, 0)
                    elif kind == b"S":
                        try:
                            desc, rows, count = fake.run(sql, params)
                        except sqlite3.Error as e:
                            self.error("42000", str(e))
                            self.send(b"Z", b"I")
                            continue
                        self.send(b"1")
                        self.send(b"2")
                        if desc:
                            cols = []
                            for i, d in enumerate(desc):
                                v = next((r[i] for r in rows if r[i] is not None), None)
                                oid = 20 if isinstance(v, int) else 701 if isinstance(v, float) else 25
                                cols.append(d[0].encode() + b"\0" + struct.pack("!IhIhih", 0, 0, oid, -1, -1, 0))
                            self.send(b"T", struct.pack("!H", len(cols)) + b"".join(cols))
                            for r in rows:
                                vals = b"".join(struct.pack("!i", -1) if v is None else
                                                struct.pack("!i", len(str(v).encode())) + str(v).encode() for v in r)
                                self.send(b"D", struct.pack("!H", len(r)) + vals)
                            tag = f"SELECT {len(rows)}"
                        else:
                            self.send(b"n")
                            verb = sql.split()[0].upper()
                            tag = {"INSERT": f"INSERT 0 {count}", "UPDATE": f"UPDATE {count}",
                                   "DELETE": f"DELETE {count}"}.get(verb, verb)
                        self.send(b"C", tag.encode() + b"\0")
                        self.send(b"Z", b"I")

        srv = socketserver.ThreadingTCPServer(("127.0.0.1", 0), H)
        srv.daemon_threads = True
        threading.Thread(target=srv.serve_forever, daemon=True).start()
        return srv


def _exercise(led):
    """The same calls on any ledger; returns everything read back."""
    out = {}
    led.insert_job("j1", "2026-01-01T00:00:00Z", {"prompt": "hi", "n": 3}, {"fp": 1}, "ph", "fh", "idem-1", "QUEUED")
    led.insert_job("j2", "2026-01-01T00:00:00Z", {"prompt": "yo"}, {"fp": 2}, "ph2", "fh", None, "QUEUED", org_id="acme")
    led.update_status("j1", "SUCCEEDED")
    out["job"] = led.get_job("j1")
    out["verify"] = led.verify_job("j1")
    out["list"] = [j["job_id"] for j in led.list_jobs(10)]  # same created_at: insertion order decides
    out["list_acme"] = [j["job_id"] for j in led.list_jobs(10, org_id="acme")]
    out["by_fp"] = led.find_job_by_fingerprint("fh", "acme")
    out["by_idem"] = led.find_job_by_idempotency("idem-1")
    led.insert_run("r1", "j1", "t0", "t1", 0, "m", "e", "o", "l")
    led.insert_run("r2", "j1", "t0", "t1", 1, "m2", "e2", "o2", "l2")
    out["run"] = led.get_latest_run("j1")
    led.insert_snapshot("s1", "j1", "fh", "/p/a", "t1")
    led.insert_snapshot("s1", "j1", "fh", "/p/b", "t2")  # replaces
    out["snap"] = led.get_snapshot_for_job("j1")
    for i in range(4):
        led.upsert_snapshot_location("fh", f"s{i}", "default", "node0", "w0", f"/p/{i}", 1 << 33, "t", f"u{i}")
    led.upsert_snapshot_location("fh", "s0", "default", "node0", "w9", "/p/0b", 7, "t", "u9")
    led.mark_snapshot_location_used("fh", "default", "node0", "s1", "u8")
    out["locs"] = led.list_snapshot_locations("fh", "default")
    out["pruned"] = led.prune_snapshot_locations(2)
    out["locs_after"] = [r["snapshot_id"] for r in led.list_snapshot_locations("fh", "default")]
    led.create_api_key("k1", "hash1", "acme", "t", 1000, 10, "{}")
    out["revoke"] = (led.revoke_api_key("k1", "t2"), led.revoke_api_key("k1", "t3"))
    out["key"] = led.get_api_key_by_hash("hash1")
    out["keys"] = led.list_api_keys("acme")
    led.upsert_replay_governance("fh", 1, "neg_roi", "t", 1767225600.123456, 3, 0, 0, "t")
    led.upsert_replay_governance("fh", 0, None, None, 0.0, 0, 0, 0, "t2")
    out["gov"] = led.get_replay_governance("fh")
    led.upsert_spec_governance("fh", "acme", 1, "low_acceptance", 1767225600.5, 0, "t")
    out["spec"] = led.list_spec_governance(5, "acme")
    return out


@pytest.mark.parametrize("auth", ["scram", "md5"])
def test_postgres_ledger_matches_sqlite(auth):
    fake = _FakePg(auth=auth)
    srv = fake.serve()
    try:
        pg = PostgresLedger(f"postgresql://korith:s3cret@127.0.0.1:{srv.server_address[1]}/ledger")
        got = _exercise(pg)
        want = _exercise(SqliteLedger(":memory:"))
        assert got == want
        assert got["list"] == ["j2", "j1"] and got["pruned"] == 2 and got["revoke"] == (True, False)
        assert got["gov"]["replay_disabled"] == 0 and got["spec"][0]["cooldown_until"] == 1767225600.5
        assert any("ON CONFLICT (snapshot_id) DO UPDATE" in s for s in fake.statements)
        assert all("?" not in s for s in fake.statements)
        pg.close()
    finally:
        srv.shutdown()
        srv.server_close()


def test_postgres_wrong_password_and_build_ledger(monkeypatch, tmp_path):
    fake = _FakePg()
    srv = fake.serve()
    try:
        with pytest.raises(PgError) as e:
            PostgresLedger(f"postgresql://korith:nope@127.0.0.1:{srv.server_address[1]}/ledger")
        assert e.value.code == "28P01"
        monkeypatch.setenv("KORITH_LEDGER_BACKEND", "postgres")
        monkeypatch.setenv("KORITH_LEDGER_DSN", f"postgresql://korith:s3cret@127.0.0.1:{srv.server_address[1]}/x")
        assert isinstance(build_ledger(), PostgresLedger)
        monkeypatch.setenv("KORITH_LEDGER_BACKEND", "sqlite")
        led = build_ledger(str(tmp_path / "d" / "ledger.sqlite"))
        assert type(led) is SqliteLedger
    finally:
        srv.shutdown()
        srv.server_close()


def test_translate():
    assert translate("SELECT * FROM jobs WHERE a=? AND b=? LIMIT ?") == "SELECT * FROM jobs WHERE a=$1 AND b=$2 LIMIT $3"
    t = translate("INSERT OR REPLACE INTO spec_governance VALUES (?,?,?,?,?,?,?)")
    assert t.startswith("INSERT INTO spec_governance VALUES ($1,$2,$3,$4,$5,$6,$7) ON CONFLICT (fingerprint_hash)")
    assert "org_id=EXCLUDED.org_id" in t and "fingerprint_hash=EXCLUDED" not in t
