"""On-disk formats: the AMFK direct-KV blob and the ``amf_index.bin`` index.

AMFK blob (reference: core/amf_direct_kv.h:35-72, amf_kv_manager.py:46-58)::

    header  <IIIIIIII QQQ>  56 B   magic 0x414D464B "AMFK", version 1, n_layers,
                                   n_tokens, n_kv_heads, head_dim, dtype, reserved,
                                   total_kv_bytes, model_hash, prefix_hash
    layers  n_layers x <QQQQ> 32 B  k_offset, k_bytes, v_offset, v_bytes
                                   (offsets relative to the payload start)
    payload                         per layer: K bytes then V bytes

K and V of one layer are the prefix's pages in ``[n_pages, n_kv_heads, page, head_dim]``
order. dtype tags 0 f16, 1 f32, 2 bf16 and 3 fp8 are the reference's. Tags 4 and 5
are this framework's extension for compressed pool pages:

* 4 ``fp8_block``: e4m3 bytes ``[n_pages, H, page, D]`` followed by one fp32 scale
  per (page, head) -- FP8 with one scale per KV block.
* 5 ``int4_g64``: packed nibbles ``[n_pages, H, page, D/2]`` followed by
  ``[n_pages, H, page, D/64, 2]`` fp16 (scale, minimum) -- asymmetric INT4, groups of
  64 along head_dim.

Index (reference: core/amf_store.cpp:36-110, :469-776): a 24-byte header
``<IIQQ>`` (magic "AMF1", version, count, checksum) then ``count`` records of 232 B
(v9) or 224 B (v8, no tenant hash in the key); checksum = FNV-1a64 over the header
with checksum 0 followed by the record bytes. The C++ store in ``_native`` is the
writer used at run time; the pure-Python codec here is an independent
implementation of the same layout used to cross-check it.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field
from typing import List, Tuple

AMFK_MAGIC = 0x414D464B
AMFK_VERSION = 1
AMFK_HEADER = struct.Struct("<IIIIIIIIQQQ")
AMFK_LAYER = struct.Struct("<QQQQ")
assert AMFK_HEADER.size == 56 and AMFK_LAYER.size == 32

DTYPE_F16, DTYPE_F32, DTYPE_BF16, DTYPE_F8 = 0, 1, 2, 3
DTYPE_FP8_BLOCK, DTYPE_INT4_G64 = 4, 5

INDEX_MAGIC = 0x31464D41
INDEX_VERSION = 9
INDEX_HEADER = struct.Struct("<IIQQ")
_KEY_V9 = "QQQIIIIQQ"
_KEY_V8 = "QQIIIIQQ"
_BODY = "QIIQQdddQQQQQQIIQQQQQQQB7x"
RECORD_V9 = struct.Struct("<" + _KEY_V9 + _BODY)
RECORD_V8 = struct.Struct("<" + _KEY_V8 + _BODY)
assert INDEX_HEADER.size == 24 and RECORD_V9.size == 232 and RECORD_V8.size == 224

_KEY_FIELDS_V9 = ["model_hash", "tenant_hash", "prefix_hash", "n_ctx", "kv_version",
                  "rope_base_bits", "rope_scale_bits", "sampling_hash", "rng_hash"]
_BODY_FIELDS = ["entry_model_hash", "prefix_len", "_r1", "seen_count", "restore_count",
                "ema_saved_ms", "ema_restore_ms", "ema_roi", "failure_count", "block_count",
                "saved_ms", "hit_count", "last_used", "last_hit_ms", "low_roi_hits", "_r2",
                "kv_size", "last_access_time_ms", "access_count", "stored_at_ms",
                "expires_at_ms", "size_bytes", "kv_checksum", "state"]


def _fnv(data: bytes, h: int = 1469598103934665603) -> int:
    from .._native_loader import native

    return int(native().fnv1a_bytes(data, h))


@dataclass
class AmfkHeader:
    n_layers: int
    n_tokens: int
    n_kv_heads: int
    head_dim: int
    dtype: int
    total_kv_bytes: int
    model_hash: int = 0
    prefix_hash: int = 0
    magic: int = AMFK_MAGIC
    version: int = AMFK_VERSION
    layers: List[Tuple[int, int, int, int]] = field(default_factory=list)

    @property
    def payload_offset(self) -> int:
        return AMFK_HEADER.size + AMFK_LAYER.size * self.n_layers


def encode_amfk_header(h: AmfkHeader) -> bytes:
    out = AMFK_HEADER.pack(h.magic, h.version, h.n_layers, h.n_tokens, h.n_kv_heads, h.head_dim,
                           h.dtype, 0, h.total_kv_bytes, h.model_hash, h.prefix_hash)
    for rec in h.layers:
        out += AMFK_LAYER.pack(*rec)
    return out


def decode_amfk_header(blob: bytes | memoryview) -> AmfkHeader:
    if len(blob) < AMFK_HEADER.size:
        raise ValueError("AMFK blob shorter than its header")
    (magic, version, n_layers, n_tokens, n_kv_heads, head_dim, dtype, _r, total,
     model_hash, prefix_hash) = AMFK_HEADER.unpack_from(blob, 0)
    if magic != AMFK_MAGIC:
        raise ValueError(f"bad AMFK magic {magic:#x}")
    if version != AMFK_VERSION:
        raise ValueError(f"unsupported AMFK version {version}")
    need = AMFK_HEADER.size + AMFK_LAYER.size * n_layers
    if len(blob) < need:
        raise ValueError("AMFK layer table truncated")
    layers = [AMFK_LAYER.unpack_from(blob, AMFK_HEADER.size + i * AMFK_LAYER.size) for i in range(n_layers)]
    h = AmfkHeader(n_layers, n_tokens, n_kv_heads, head_dim, dtype, total, model_hash, prefix_hash,
                   magic, version, layers)
    if len(blob) < h.payload_offset + total:
        raise ValueError("AMFK payload truncated")
    for ko, kb, vo, vb in layers:
        if ko + kb > total or vo + vb > total:
            raise ValueError("AMFK layer record points outside the payload")
    return h


def is_amfk(blob: bytes | memoryview) -> bool:
    return len(blob) >= 4 and struct.unpack_from("<I", blob, 0)[0] == AMFK_MAGIC


def page_bytes(dtype: int, n_kv_heads: int, page: int, head_dim: int) -> int:
    """Bytes of one K (or V) page of one layer in the given AMFK dtype."""
    vals = n_kv_heads * page * head_dim
    if dtype in (DTYPE_F16, DTYPE_BF16):
        return 2 * vals
    if dtype == DTYPE_F32:
        return 4 * vals
    if dtype == DTYPE_F8:
        return vals
    if dtype == DTYPE_FP8_BLOCK:
        return vals + 4 * n_kv_heads
    if dtype == DTYPE_INT4_G64:
        return vals // 2 + 4 * n_kv_heads * page * math.ceil(head_dim / 64)
    raise ValueError(f"unknown AMFK dtype {dtype}")


# -------------------------------------------------------------------------- index codec
def encode_index(entries: List[dict]) -> bytes:
    body = b"".join(_pack_record(e) for e in entries)
    hdr0 = INDEX_HEADER.pack(INDEX_MAGIC, INDEX_VERSION, len(entries), 0)
    checksum = _fnv(hdr0 + body)
    return INDEX_HEADER.pack(INDEX_MAGIC, INDEX_VERSION, len(entries), checksum) + body


def _pack_record(e: dict) -> bytes:
    vals = [int(e.get(k, 0)) for k in _KEY_FIELDS_V9]
    for k in _BODY_FIELDS:
        if k.startswith("_r"):
            vals.append(0)
        elif k.startswith("ema_"):
            vals.append(float(e.get(k, float("nan"))))
        elif k == "entry_model_hash":
            vals.append(int(e.get(k, e.get("model_hash", 0))))
        else:
            vals.append(int(e.get(k, 0)))
    return RECORD_V9.pack(*vals)


def decode_index(data: bytes) -> Tuple[int, List[dict]]:
    """Returns (version, entries); raises ValueError on any corruption."""
    if len(data) < INDEX_HEADER.size:
        raise ValueError("index shorter than its header")
    magic, version, count, checksum = INDEX_HEADER.unpack_from(data, 0)
    if magic != INDEX_MAGIC:
        raise ValueError("bad index magic")
    if version not in (8, 9):
        raise ValueError(f"unsupported index version {version}")
    if count > (1 << 20):
        raise ValueError("index record count out of range")
    rec = RECORD_V9 if version == 9 else RECORD_V8
    end = INDEX_HEADER.size + count * rec.size
    if len(data) < end:
        raise ValueError("index truncated")
    if _fnv(INDEX_HEADER.pack(magic, version, count, 0) + data[INDEX_HEADER.size:end]) != checksum:
        raise ValueError("index checksum mismatch")
    keys = _KEY_FIELDS_V9 if version == 9 else [k for k in _KEY_FIELDS_V9 if k != "tenant_hash"]
    names = keys + _BODY_FIELDS
    out = []
    for i in range(count):
        vals = rec.unpack_from(data, INDEX_HEADER.size + i * rec.size)
        d = {k: v for k, v in zip(names, vals) if not k.startswith("_r")}
        d.setdefault("tenant_hash", 0)
        out.append(d)
    return version, out
