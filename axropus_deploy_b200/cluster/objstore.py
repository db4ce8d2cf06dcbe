"""Artifact stores: the local directory tree, and S3 / MinIO (any S3-compatible endpoint)
spoken over HTTP with SigV4 signing, no SDK.

Every store keeps the local job directory (the worker writes its files there) and
answers ``init_job / store_artifact / get_artifact``; the object store also does
``upload_job`` (every file of the job directory), ``list_artifacts`` and ``delete_artifact``.
Object keys are ``<prefix>/<org>/<job>/<artifact type>``. S3 uses virtual-host addressing
on AWS (``https://<bucket>.s3.<region>.amazonaws.com``) and path addressing on a custom
endpoint (MinIO: ``http(s)://<endpoint>/<bucket>/<key>``).

:func:`build_artifacts` picks one from ``KORITH_ARTIFACT_BACKEND`` (``local`` default, ``s3``
with ``KORITH_S3_BUCKET`` / ``KORITH_S3_PREFIX`` / optional ``KORITH_S3_ENDPOINT``, ``minio``
with ``KORITH_MINIO_ENDPOINT`` / ``_ACCESS_KEY`` / ``_SECRET_KEY`` / ``_BUCKET`` / ``_PREFIX`` /
``_SECURE``) under the local base ``KORITH_PLATFORM_ARTIFACTS``.

Reference: platform/artifacts/adapter.py (interface, local adapter), s3_store.py,
minio_store.py and platform/runtime/config.py:127-149 (selection and variables).
"""
from __future__ import annotations

import os
import urllib.parse
import xml.etree.ElementTree as ET
from pathlib import Path
from typing import Dict, List, Optional

from .observability import ArtifactStore
from .sigv4 import Credentials, SignedHttp


class LocalArtifactStore:
    def __init__(self, base_dir):
        self._store = ArtifactStore(base_dir)

    def init_job(self, job_id: str, org_id: str = "default") -> Dict[str, Path]:
        return self._store.init_job(job_id, org_id=org_id)

    def store_artifact(self, job_id: str, artifact_type: str, blob: bytes, org_id: str = "default") -> str:
        paths = self.init_job(job_id, org_id)
        if artifact_type not in paths or artifact_type == "job_dir":
            raise ValueError(f"unknown artifact type {artifact_type}")
        Path(paths[artifact_type]).write_bytes(blob)
        return str(paths[artifact_type])

    def get_artifact(self, job_id: str, artifact_type: str, org_id: str = "default") -> Optional[bytes]:
        p = self.init_job(job_id, org_id).get(artifact_type)
        return Path(p).read_bytes() if p is not None and Path(p).is_file() else None


class S3ArtifactStore(LocalArtifactStore):
    def __init__(self, base_dir, bucket: str, prefix: str = "korith", endpoint: Optional[str] = None,
                 region: Optional[str] = None, creds: Optional[Credentials] = None, http: Optional[SignedHttp] = None):
        super().__init__(base_dir)
        if not bucket:
            raise ValueError("S3 artifact store needs a bucket")
        self.bucket, self.prefix = bucket, prefix.strip("/")
        self.http = http or SignedHttp("s3", region, creds)
        if endpoint:
            self.base = endpoint.rstrip("/") + "/" + bucket  # path-style (MinIO and other S3-compatible servers)
        else:
            self.base = f"https://{bucket}.s3.{self.http.region}.amazonaws.com"

    def _key(self, job_id: str, artifact_type: str, org_id: str = "default") -> str:
        return f"{self.prefix}/{org_id}/{job_id}/{artifact_type}"

    def _url(self, key: str) -> str:
        return f"{self.base}/{urllib.parse.quote(key, safe='/-_.~')}"

    def store_artifact(self, job_id: str, artifact_type: str, blob: bytes, org_id: str = "default") -> str:
        key = self._key(job_id, artifact_type, org_id)
        st, _, body = self.http.request("PUT", self._url(key), bytes(blob))
        if st not in (200, 201):
            raise RuntimeError(f"S3 PUT {key} failed: HTTP {st} {body[:200]!r}")
        return key

    def get_artifact(self, job_id: str, artifact_type: str, org_id: str = "default") -> Optional[bytes]:
        st, _, body = self.http.request("GET", self._url(self._key(job_id, artifact_type, org_id)))
        return body if st == 200 else None

    def delete_artifact(self, job_id: str, artifact_type: str, org_id: str = "default") -> bool:
        st, _, _ = self.http.request("DELETE", self._url(self._key(job_id, artifact_type, org_id)))
        return st in (200, 204)

    def upload_job(self, job_id: str, org_id: str = "default") -> List[str]:
        """Every file of the local job directory, under its artifact type."""
        keys = []
        for kind, p in self.init_job(job_id, org_id).items():
            if kind != "job_dir" and Path(p).is_file():
                keys.append(self.store_artifact(job_id, kind, Path(p).read_bytes(), org_id))
        return keys

    def list_artifacts(self, job_id: str, org_id: str = "default") -> List[str]:
        pre = f"{self.prefix}/{org_id}/{job_id}/"
        out: List[str] = []
        token = None
        while True:
            q = {"list-type": "2", "prefix": pre}
            if token:
                q["continuation-token"] = token
            st, _, body = self.http.request("GET", f"{self.base}/?{urllib.parse.urlencode(sorted(q.items()))}")
            if st != 200:
                raise RuntimeError(f"S3 list {pre} failed: HTTP {st}")
            root = ET.fromstring(body)
            ns = root.tag[: root.tag.index("}") + 1] if root.tag.startswith("{") else ""
            out += [c.findtext(f"{ns}Key")[len(pre):] for c in root.findall(f"{ns}Contents")]
            if (root.findtext(f"{ns}IsTruncated") or "false").lower() != "true":
                return out
            token = root.findtext(f"{ns}NextContinuationToken")


def build_artifacts(base_dir=None):
    backend = os.environ.get("KORITH_ARTIFACT_BACKEND", "local").strip().lower()
    base = Path(base_dir or os.environ.get("KORITH_PLATFORM_ARTIFACTS", "./platform_data/artifacts")).resolve()
    if backend == "s3":
        return S3ArtifactStore(base, os.environ.get("KORITH_S3_BUCKET", ""), os.environ.get("KORITH_S3_PREFIX", "korith"),
                               endpoint=os.environ.get("KORITH_S3_ENDPOINT") or None)
    if backend == "minio":
        ep = os.environ.get("KORITH_MINIO_ENDPOINT", "")
        if "://" not in ep:
            secure = os.environ.get("KORITH_MINIO_SECURE", "true").lower() == "true"
            ep = ("https://" if secure else "http://") + ep
        creds = Credentials(os.environ.get("KORITH_MINIO_ACCESS_KEY", ""), os.environ.get("KORITH_MINIO_SECRET_KEY", ""))
        return S3ArtifactStore(base, os.environ.get("KORITH_MINIO_BUCKET", ""),
                               os.environ.get("KORITH_MINIO_PREFIX", "korith"), endpoint=ep, creds=creds)
    if backend != "local":
        raise ValueError(f"unknown KORITH_ARTIFACT_BACKEND {backend!r}")
    return LocalArtifactStore(base)
