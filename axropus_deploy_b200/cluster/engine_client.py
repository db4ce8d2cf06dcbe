"""ctypes client of the C ABI library (``libkorith_b200.so``) and the metadata sidecar
of KV snapshot files.

:class:`EngineClient` binds the ``korith_engine_*`` entry points with their argument
types; every call returns Python values (``None`` / ``False`` on failure, the message in
:meth:`EngineClient.last_error`). :func:`write_snapshot_metadata` /
:func:`validate_snapshot_metadata` keep a ``<snapshot>.meta.json`` beside a snapshot
(format tag, fingerprint / model / tokenizer hashes, KV layout version, context
length, size and sha256), so a snapshot fetched from another node is only replayed
into a matching engine, and a corrupted one is refused.

Reference: platform/engine/loader.py (ctypes client), platform/engine/snapshot.py:9-98
(sidecar fields and the validation order).
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

SNAPSHOT_FORMAT = "korith.kv_snapshot.v1"
DEFAULT_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "libkorith_b200.so")


class _Params(ctypes.Structure):
    _fields_ = [("n_ctx", ctypes.c_int32), ("n_batch", ctypes.c_int32), ("n_gpu", ctypes.c_int32),
                ("model_path", ctypes.c_char_p)]


class _Metrics(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in ("prefill_ms", "decode_ms", "total_ms", "restore_ms", "verify_ms",
                                               "draft_ms")] + \
               [(n, ctypes.c_int32) for n in ("tokens_out", "accepted_tokens", "rejected_tokens")]


class EngineClient:
    def __init__(self, lib_path: Optional[str] = None):
        path = lib_path or os.environ.get("KORITH_ENGINE_LIB", DEFAULT_LIB)
        if not os.path.exists(path):
            raise FileNotFoundError(f"C ABI library not built: {path}")
        lib = self.lib = ctypes.CDLL(path)
        b, i32p = ctypes.c_bool, ctypes.POINTER(ctypes.c_int32)
        sig = {
            "korith_engine_init_model": (b, [ctypes.POINTER(_Params)]),
            "korith_engine_prefill": (b, [i32p, ctypes.c_int32]),
            "korith_engine_decode_step": (b, [i32p]),
            "korith_engine_get_logits": (b, [ctypes.POINTER(ctypes.c_float), ctypes.c_int32]),
            "korith_engine_apply_kv_replay": (b, [ctypes.c_char_p, ctypes.c_size_t]),
            "korith_engine_export_snapshot": (b, [ctypes.c_char_p]),
            "korith_engine_import_snapshot": (b, [ctypes.c_char_p]),
            "korith_engine_verify_tokens": (b, [i32p, ctypes.c_int32, i32p]),
            "korith_engine_get_metrics": (None, [ctypes.POINTER(_Metrics)]),
            "korith_engine_shutdown": (None, []),
            "korith_engine_cuda_probe": (b, []),
            "korith_last_error": (ctypes.c_char_p, []),
        }
        for name, (res, args) in sig.items():
            f = getattr(lib, name)
            f.restype, f.argtypes = res, args

    @staticmethod
    def _ints(v: List[int]):
        return (ctypes.c_int32 * len(v))(*[int(x) for x in v])

    def last_error(self) -> str:
        return (self.lib.korith_last_error() or b"").decode("utf-8", "replace")

    def init_model(self, model_path: str, n_ctx: int, n_batch: int = 1, n_gpu: int = 1) -> bool:
        p = _Params(int(n_ctx), int(n_batch), int(n_gpu), model_path.encode())
        return bool(self.lib.korith_engine_init_model(ctypes.byref(p)))

    def prefill(self, tokens: List[int]) -> bool:
        return bool(tokens) and bool(self.lib.korith_engine_prefill(self._ints(tokens), len(tokens)))

    def decode_step(self) -> Optional[int]:
        t = ctypes.c_int32(-1)
        return int(t.value) if self.lib.korith_engine_decode_step(ctypes.byref(t)) else None

    def logits(self, n_vocab: int) -> Optional[List[float]]:
        buf = (ctypes.c_float * n_vocab)()
        return list(buf) if self.lib.korith_engine_get_logits(buf, n_vocab) else None

    def apply_kv_replay(self, blob: bytes) -> bool:
        return bool(self.lib.korith_engine_apply_kv_replay(blob, len(blob)))

    def export_snapshot(self, path: str) -> bool:
        return bool(self.lib.korith_engine_export_snapshot(str(path).encode()))

    def import_snapshot(self, path: str) -> bool:
        return bool(self.lib.korith_engine_import_snapshot(str(path).encode()))

    def verify(self, proposed: List[int]) -> int:
        acc = ctypes.c_int32(0)
        ok = self.lib.korith_engine_verify_tokens(self._ints(proposed), len(proposed), ctypes.byref(acc))
        return int(acc.value) if ok else -1

    def metrics(self) -> Dict[str, Any]:
        m = _Metrics()
        self.lib.korith_engine_get_metrics(ctypes.byref(m))
        return {n: getattr(m, n) for n, _ in _Metrics._fields_}

    def cuda_probe(self) -> bool:
        return bool(self.lib.korith_engine_cuda_probe())

    def shutdown(self) -> None:
        self.lib.korith_engine_shutdown()


# ---------------------------------------------------------------------- snapshot sidecars
def snapshot_meta_path(snapshot_path) -> Path:
    p = Path(snapshot_path)
    return p.with_name(p.name + ".meta.json")


def snapshot_checksum(snapshot_path) -> str:
    h = hashlib.sha256()
    with Path(snapshot_path).open("rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def write_snapshot_metadata(snapshot_path, *, fingerprint_hash: str, model_hash: str, tokenizer_hash: str,
                            backend_id: str, n_ctx: int, kv_layout_version: str, created_at: str) -> Path:
    snap = Path(snapshot_path)
    meta = {"format": SNAPSHOT_FORMAT, "fingerprint_hash": fingerprint_hash, "model_hash": model_hash,
            "tokenizer_hash": tokenizer_hash, "backend_id": backend_id, "n_ctx": int(n_ctx),
            "kv_layout_version": kv_layout_version, "size_bytes": snap.stat().st_size if snap.exists() else 0,
            "checksum_sha256": snapshot_checksum(snap) if snap.exists() else "", "created_at": created_at}
    out = snapshot_meta_path(snap)
    out.write_text(json.dumps(meta, indent=2), encoding="utf-8")
    return out


def validate_snapshot_metadata(snapshot_path, *, fingerprint_hash: str, model_hash: str, tokenizer_hash: str,
                               kv_layout_version: str, n_ctx: int) -> Tuple[bool, str, Optional[Dict[str, Any]]]:
    """(ok, reason, meta). Checks run cheapest first; the checksum last."""
    snap = Path(snapshot_path)
    if not snap.exists():
        return False, "snapshot_missing", None
    try:
        meta = json.loads(snapshot_meta_path(snap).read_text(encoding="utf-8"))
    except (OSError, ValueError):
        return False, "snapshot_meta_missing", None
    checks = (("format", SNAPSHOT_FORMAT, "snapshot_meta_format_invalid"),
              ("fingerprint_hash", fingerprint_hash, "snapshot_fingerprint_mismatch"),
              ("model_hash", model_hash, "snapshot_model_mismatch"),
              ("tokenizer_hash", tokenizer_hash, "snapshot_tokenizer_mismatch"),
              ("kv_layout_version", kv_layout_version, "snapshot_layout_mismatch"))
    for key, want, reason in checks:
        if str(meta.get(key, "")) != str(want):
            return False, reason, meta
    if int(meta.get("n_ctx", 0) or 0) != int(n_ctx):
        return False, "snapshot_ctx_mismatch", meta
    if not str(meta.get("checksum_sha256", "")).strip():
        return False, "snapshot_checksum_missing", meta
    if snapshot_checksum(snap) != meta["checksum_sha256"]:
        return False, "snapshot_checksum_mismatch", meta
    return True, "ok", meta
