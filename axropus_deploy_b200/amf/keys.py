"""AMF key namespaces and file naming.

Two independent key namespaces exist, exactly as in the reference:

* **Disk store keys** (FNV-1a 64): token-prefix hash ``h ^= u32(tok); h *= prime``
  over the whole prompt prefix, tenant/model hashes over bytes, and the 9-field
  ``AmfKey`` that names the entry files (core/amf_store.cpp:27-28, :118-129,
  :778-793).
* **G1 pool keys** (sha256): ``sha256(le32 tokens)[:16]`` as 16 hex characters
  (korith_vllm_ext/tiered_router.py:85-95, amf_kv_connector.py:66-71). The pool
  uses the 64-bit integer of those 16 hex digits; its owner GPU is ``key % world``.

Entry basenames are written in the C++ spelling (``%08x`` for n_ctx, kv_version
and the rope bits) and parsed in both the C++ and the Python-writer spelling
(decimal, amf_kv_manager.py:133-135).
"""
from __future__ import annotations

import hashlib
import re
import struct
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from .._native_loader import native

FNV_OFFSET = 1469598103934665603
FNV_PRIME = 1099511628211
_MASK = (1 << 64) - 1
# Engine constants for the deterministic-replay key fields (core/engine.cpp:673-705).
RNG_HASH_CONST = 0x4B4F524954485F30  # "KORITH_0"


def _as_i32(tokens: Sequence[int]) -> np.ndarray:
    a = np.asarray(tokens)
    if a.dtype != np.int32:
        a = (a.astype(np.int64) & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
    return np.ascontiguousarray(a)


def fnv1a_bytes(data: bytes, h: int = FNV_OFFSET) -> int:
    return int(native().fnv1a_bytes(data, h))


def amf_hash_tokens(tokens: Sequence[int]) -> int:
    """FNV-1a over token ids (each id xor-ed in as one 32-bit value)."""
    return int(native().fnv1a_tokens(_as_i32(tokens)))


def amf_prefix_hashes(tokens: Sequence[int]) -> np.ndarray:
    """Rolling hashes: element i is the hash of tokens[:i+1]."""
    return native().prefix_hashes(_as_i32(tokens))


def amf_hash_tenant_id(tenant_id: str) -> int:
    return FNV_OFFSET if not tenant_id else fnv1a_bytes(tenant_id.encode("utf-8"))


def amf_hash_model_file(path: str) -> int:
    """FNV-1a over a model file's bytes (0 if missing), streamed in 1 MiB chunks."""
    h = FNV_OFFSET
    try:
        with open(path, "rb") as f:
            while True:
                chunk = f.read(1 << 20)
                if not chunk:
                    break
                h = fnv1a_bytes(chunk, h)
    except FileNotFoundError:
        return 0
    return h


def amf_hash_model_name(name: str) -> int:
    """Model identity for random-init / hub models that have no single weight file."""
    return fnv1a_bytes(("model:" + name).encode("utf-8"))


def amf_float_bits(v: float) -> int:
    return struct.unpack("<I", struct.pack("<f", v))[0]


def hash_u64_step(h: int, v: int) -> int:
    return ((h ^ (v & _MASK)) * FNV_PRIME) & _MASK


def sampling_hash(bench_mode: int = 0, bench_min: int = 0, scheme: int = 1) -> int:
    """Deterministic-sampling identity folded into the key (scheme, bench mode, min)."""
    h = FNV_OFFSET
    for v in (scheme, bench_mode, bench_min):
        h = hash_u64_step(h, v)
    return h


def pool_key(tokens: Sequence[int]) -> str:
    """G1 pool / connector key: sha256 over little-endian int32 ids, 16 hex chars."""
    return hashlib.sha256(_as_i32(tokens).astype("<i4").tobytes()).hexdigest()[:16]


def pool_key_int(key: str) -> int:
    v = int(key, 16)
    return v if v != 0 else 1  # 0 marks an empty directory slot


def pool_key2(tokens: Sequence[int]) -> int:
    """Independent 64-bit check hash stored beside the pool key (collision guard)."""
    return amf_hash_tokens(tokens) or 1


def owner_of(key: str, world: int) -> int:
    return pool_key_int(key) % max(1, world)


@dataclass(frozen=True)
class AmfContext:
    model_hash: int = 0
    tenant_hash: int = FNV_OFFSET
    n_ctx: int = 0
    kv_version: int = 0
    rope_base_bits: int = 0
    rope_scale_bits: int = 0
    sampling_hash: int = 0
    rng_hash: int = 0

    def as_dict(self) -> dict:
        return dict(self.__dict__)


def entry_basename(model_hash: int, tenant_hash: int, prefix_hash: int, n_ctx: int,
                   kv_version: int, rope_base_bits: int, rope_scale_bits: int,
                   sampling_hash_: int, rng_hash: int, *, python_spelling: bool = False) -> str:
    if python_spelling:
        mid = f"{n_ctx}_{kv_version}_{rope_base_bits}_{rope_scale_bits}"
    else:
        mid = f"{n_ctx:08x}_{kv_version:08x}_{rope_base_bits:08x}_{rope_scale_bits:08x}"
    return (f"amf_{model_hash:016x}_{tenant_hash:016x}_{prefix_hash:016x}_{mid}"
            f"_{sampling_hash_:016x}_{rng_hash:016x}")


_NAME_RE = re.compile(
    r"^amf_([0-9a-f]{16})_([0-9a-f]{16})_([0-9a-f]{16})_([0-9a-f]+)_([0-9a-f]+)_([0-9a-f]+)_([0-9a-f]+)"
    r"_([0-9a-f]{16})_([0-9a-f]{16})$")


def parse_basename(name: str) -> Optional[dict]:
    """Parse either spelling. The C++ spelling is exactly 8 hex digits per 32-bit
    field; anything else is read as the Python writer's decimal spelling."""
    m = _NAME_RE.match(name)
    if not m:
        return None
    g = m.groups()
    mid = g[3:7]
    cxx = all(len(x) == 8 for x in mid)
    try:
        vals = [int(x, 16) if cxx else int(x, 10) for x in mid]
    except ValueError:
        return None
    return {
        "model_hash": int(g[0], 16), "tenant_hash": int(g[1], 16), "prefix_hash": int(g[2], 16),
        "n_ctx": vals[0], "kv_version": vals[1], "rope_base_bits": vals[2], "rope_scale_bits": vals[3],
        "sampling_hash": int(g[7], 16), "rng_hash": int(g[8], 16), "spelling": "cxx" if cxx else "python",
    }
