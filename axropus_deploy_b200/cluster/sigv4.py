"""AWS Signature Version 4 request signing and a small signed HTTP client, for the S3 /
MinIO artifact store and the SQS queue without an AWS SDK.

The signature follows AWS's published SigV4 algorithm: a canonical request (method, URI
path, sorted query, sorted lower-case headers, signed header list, payload sha256), the
string to sign ``AWS4-HMAC-SHA256 / timestamp / scope / sha256(canonical request)``, and
an HMAC-SHA256 chain ``date -> region -> service -> "aws4_request"`` from ``"AWS4" + secret``.
Credentials come from the arguments or ``AWS_ACCESS_KEY_ID`` / ``AWS_SECRET_ACCESS_KEY`` /
``AWS_SESSION_TOKEN``; the region from ``AWS_REGION`` / ``AWS_DEFAULT_REGION``.

Reference: platform/artifacts/s3_store.py and platform/queue/sqs_queue.py (they sign
through boto3; this module replaces that dependency).
"""
from __future__ import annotations

import datetime as _dt
import hashlib
import hmac
import http.client
import os
import urllib.parse
from dataclasses import dataclass
from typing import Dict, Optional, Tuple


def _h(key: bytes, msg: str) -> bytes:
    return hmac.new(key, msg.encode("utf-8"), hashlib.sha256).digest()


def signing_key(secret: str, date: str, region: str, service: str) -> bytes:
    k = _h(("AWS4" + secret).encode("utf-8"), date)
    k = _h(k, region)
    k = _h(k, service)
    return _h(k, "aws4_request")


def _quote(s: str, safe: str = "-_.~") -> str:
    return urllib.parse.quote(s, safe=safe)


@dataclass
class Credentials:
    access_key: str
    secret_key: str
    token: Optional[str] = None

    @classmethod
    def from_env(cls) -> "Credentials":
        return cls(os.environ.get("AWS_ACCESS_KEY_ID", ""), os.environ.get("AWS_SECRET_ACCESS_KEY", ""),
                   os.environ.get("AWS_SESSION_TOKEN") or None)


def sign(method: str, url: str, headers: Dict[str, str], body: bytes, creds: Credentials, region: str,
         service: str, now: Optional[_dt.datetime] = None, unsigned_payload: bool = False) -> Dict[str, str]:
    """Headers of the signed request (the given ones plus host, x-amz-date, x-amz-content-sha256
    for S3, x-amz-security-token when there is a session token, and Authorization)."""
    u = urllib.parse.urlsplit(url)
    t = (now or _dt.datetime.now(_dt.timezone.utc)).strftime("%Y%m%dT%H%M%SZ")
    date = t[:8]
    payload_hash = "UNSIGNED-PAYLOAD" if unsigned_payload else hashlib.sha256(body or b"").hexdigest()
    out = dict(headers)
    out["host"] = u.netloc
    out["x-amz-date"] = t
    if service == "s3":
        out["x-amz-content-sha256"] = payload_hash
    if creds.token:
        out["x-amz-security-token"] = creds.token
    canon_headers = sorted((k.lower().strip(), " ".join(str(v).strip().split())) for k, v in out.items())
    signed = ";".join(k for k, _ in canon_headers)
    q = urllib.parse.parse_qsl(u.query, keep_blank_values=True)
    canon_query = "&".join(f"{_quote(k)}={_quote(v)}" for k, v in sorted(q))
    path = u.path or "/"
    # S3 signs the path as sent; every other service signs it URI-encoded twice
    canon_path = path if service == "s3" else "/".join(_quote(_quote(p)) for p in path.split("/"))
    creq = "\n".join([method.upper(), canon_path, canon_query, "".join(f"{k}:{v}\n" for k, v in canon_headers),
                      signed, payload_hash])
    scope = f"{date}/{region}/{service}/aws4_request"
    sts = "\n".join(["AWS4-HMAC-SHA256", t, scope, hashlib.sha256(creq.encode("utf-8")).hexdigest()])
    sig = hmac.new(signing_key(creds.secret_key, date, region, service), sts.encode("utf-8"),
                   hashlib.sha256).hexdigest()
    out["Authorization"] = (f"AWS4-HMAC-SHA256 Credential={creds.access_key}/{scope}, SignedHeaders={signed}, "
                            f"Signature={sig}")
    return out


class SignedHttp:
    """One signed request at a time over a fresh connection (no pooling: artifact and queue
    calls are infrequent next to the work they describe)."""

    def __init__(self, service: str, region: Optional[str] = None, creds: Optional[Credentials] = None,
                 timeout_s: float = 30.0):
        self.service = service
        self.region = region or os.environ.get("AWS_REGION") or os.environ.get("AWS_DEFAULT_REGION") or "us-east-1"
        self.creds = creds or Credentials.from_env()
        self.timeout_s = timeout_s

    def request(self, method: str, url: str, body: bytes = b"",
                headers: Optional[Dict[str, str]] = None) -> Tuple[int, Dict[str, str], bytes]:
        u = urllib.parse.urlsplit(url)
        h = sign(method, url, dict(headers or {}), body, self.creds, self.region, self.service)
        conn_cls = http.client.HTTPSConnection if u.scheme == "https" else http.client.HTTPConnection
        conn = conn_cls(u.hostname, u.port, timeout=self.timeout_s)
        try:
            target = (u.path or "/") + (("?" + u.query) if u.query else "")
            conn.request(method, target, body=body or None, headers=h)
            r = conn.getresponse()
            return r.status, {k.lower(): v for k, v in r.getheaders()}, r.read()
        finally:
            conn.close()
