"""AMF disk store (native) and on-disk formats: hashing goldens, index codec parity
between the C++ writer and an independent Python codec, and the store scenarios of
the reference's C++ store tests (basic lookup, tenant isolation, watermark eviction,
TTL, model mismatch, persistence, disk guard, prewarm, version reset)."""
import os
import struct
import time

import numpy as np
import pytest

from axropus_deploy_b200._native_loader import native
from axropus_deploy_b200.amf import formats, keys

U64 = (1 << 64) - 1


def _golden_123():
    h = keys.FNV_OFFSET
    for t in (1, 2, 3):
        h = ((h ^ t) * keys.FNV_PRIME) & U64
    return h


def test_fnv_goldens():
    assert keys.amf_hash_tokens([]) == keys.FNV_OFFSET
    assert keys.amf_hash_tokens([1, 2, 3]) == _golden_123()
    assert keys.amf_hash_tokens([0]) == (keys.FNV_OFFSET * keys.FNV_PRIME) & U64
    assert keys.amf_hash_tenant_id("") == keys.FNV_OFFSET
    assert keys.amf_hash_tenant_id("nebius") not in (0, keys.FNV_OFFSET)
    assert keys.amf_float_bits(1.0) == 0x3F800000 and keys.amf_float_bits(0.0) == 0
    ph = keys.amf_prefix_hashes([1, 2, 3])
    assert int(ph[-1]) == _golden_123() and len(ph) == 3
    # negative ids hash as their uint32 value
    assert keys.amf_hash_tokens([-1]) == ((keys.FNV_OFFSET ^ 0xFFFFFFFF) * keys.FNV_PRIME) & U64


def test_basename_spellings():
    cxx = keys.entry_basename(0xDEADBEEFCAFEBABE, 0x0102030405060708, 0xAABBCCDD11223344, 32768, 1,
                              keys.amf_float_bits(10000.0), keys.amf_float_bits(1.0), 0, 0)
    py = keys.entry_basename(0xDEADBEEFCAFEBABE, 0x0102030405060708, 0xAABBCCDD11223344, 32768, 1,
                             keys.amf_float_bits(10000.0), keys.amf_float_bits(1.0), 0, 0, python_spelling=True)
    assert "_00008000_00000001_" in cxx and "_32768_1_" in py
    a, b = keys.parse_basename(cxx), keys.parse_basename(py)
    assert a["spelling"] == "cxx" and b["spelling"] == "python"
    for k in ("model_hash", "tenant_hash", "prefix_hash", "n_ctx", "kv_version", "rope_base_bits"):
        assert a[k] == b[k]


def _entry(i):
    return {"model_hash": 7, "tenant_hash": 9, "prefix_hash": 1000 + i, "n_ctx": 8192, "kv_version": 1,
            "rope_base_bits": 3, "rope_scale_bits": 4, "sampling_hash": 5, "rng_hash": 6, "prefix_len": 64 + i,
            "seen_count": i, "ema_saved_ms": 1.5 * i, "ema_restore_ms": float("nan"), "ema_roi": 2.0,
            "kv_size": 100 * i, "size_bytes": 100 * i, "kv_checksum": 12345 + i, "state": 2,
            "access_count": i, "stored_at_ms": 10 ** 12 + i}


def test_index_codec_parity():
    n = native()
    for i in range(3):
        e = _entry(i)
        cxx = n.encode_record_v9(e)
        py = formats.RECORD_V9.pack(*[0] * 0, *formats._pack_record(e)) if False else formats._pack_record(e)
        assert cxx == py
        back = n.decode_record(cxx, 9)
        assert back["prefix_hash"] == e["prefix_hash"] and back["prefix_len"] == e["prefix_len"]
    data = formats.encode_index([_entry(i) for i in range(4)])
    ver, entries = formats.decode_index(data)
    assert ver == 9 and len(entries) == 4 and entries[2]["kv_checksum"] == 12347
    bad = bytearray(data)
    bad[-3] ^= 0xFF
    with pytest.raises(ValueError):
        formats.decode_index(bytes(bad))


def _ctx(tenant="__shared__", **kw):
    c = keys.AmfContext(model_hash=0x1111, tenant_hash=keys.amf_hash_tenant_id(tenant), n_ctx=4096,
                        sampling_hash=0x2222, rng_hash=0x5555)
    d = c.as_dict()
    d.update(kw)
    return d


def _store(tmp_path, **cfg):
    s = native().AmfStore()
    conf = {"min_tokens": 2, "max_bytes": 1 << 20, "storage_budget_bytes": 1 << 20}
    conf.update(cfg)
    assert s.init(str(tmp_path), conf)
    return s


def test_basic_lookup_and_key_fields(tmp_path):
    s = _store(tmp_path)
    toks = np.array([1, 2, 3, 4], dtype=np.int32)
    assert s.store_entry(_ctx(), toks, b"k" * 16, 5)
    assert s.find_longest_prefix(_ctx(), toks)[0] == "hit"
    assert s.find_longest_prefix(_ctx(sampling_hash=0x3333), toks)[0] != "hit"
    assert s.find_longest_prefix(_ctx(rng_hash=0x4444), toks)[0] != "hit"
    # longest prefix of a longer prompt
    r, e = s.find_longest_prefix(_ctx(), np.array([1, 2, 3, 4, 9, 9], dtype=np.int32))
    assert r == "hit" and e["prefix_len"] == 4
    assert s.find_longest_prefix(_ctx(), np.array([1], dtype=np.int32))[0] == "short_prefix"
    # the index file is the C++ layout the Python codec reads
    ver, ents = formats.decode_index(open(os.path.join(tmp_path, "amf_index.bin"), "rb").read())
    assert ver == 9 and ents[0]["prefix_len"] == 4


def test_tenant_isolation(tmp_path):
    s = _store(tmp_path)
    toks = np.array([7, 8, 9, 10], dtype=np.int32)
    assert s.store_entry(_ctx("tenant-a"), toks, b"x" * 16, 1)
    assert s.find_longest_prefix(_ctx("tenant-a"), toks)[0] == "hit"
    assert s.find_longest_prefix(_ctx("tenant-b"), toks)[0] != "hit"


def test_watermark_eviction_lfu(tmp_path):
    s = _store(tmp_path, max_bytes=100, storage_budget_bytes=100, eviction_watermark=0.9, policy="lfu",
               hot_ttl_ms=60000, warm_ttl_ms=120000)
    c = _ctx()
    assert s.store_entry(c, np.array([11, 12], dtype=np.int32), b"a" * 40, 1)
    assert s.store_entry(c, np.array([21, 22], dtype=np.int32), b"b" * 40, 1)
    r, e = s.find_longest_prefix(c, np.array([11, 12], dtype=np.int32))
    s.note_hit(e, 2, 1, 10)  # make {11,12} more frequently used
    assert s.store_entry(c, np.array([31, 32], dtype=np.int32), b"c" * 40, 1)  # 120 > 90 -> evict
    assert s.find_longest_prefix(c, np.array([11, 12], dtype=np.int32))[0] == "hit"
    assert s.find_longest_prefix(c, np.array([21, 22], dtype=np.int32))[0] != "hit"
    assert s.stats()["evictions"] == 1


def test_ttl_expiry_and_adaptive_ttl(tmp_path):
    s = _store(tmp_path, default_ttl_ms=1, max_ttl_ms=1)
    c = _ctx()
    toks = np.array([5, 6, 7], dtype=np.int32)
    assert s.store_entry(c, toks, b"z" * 8, 1)
    time.sleep(0.01)
    assert s.find_longest_prefix(c, toks)[0] != "hit"
    assert s.entry_count == 0
    s2 = _store(tmp_path / "b", default_ttl_ms=1000, max_ttl_ms=10_000)
    assert s2.store_entry(c, toks, b"z" * 8, 1)
    r, e = s2.find_longest_prefix(c, toks)
    for _ in range(3):
        s2.note_hit(e, 3, 1, 5)
    e2 = s2.entries()[0]
    # adaptive TTL: default * (1 + log2(access_count)) = 1000 * (1 + log2 3)
    assert e2["expires_at_ms"] - e2["last_access_time_ms"] == 2584
    assert e2["access_count"] == 3


def test_model_mismatch_evicts(tmp_path):
    s = _store(tmp_path)
    toks = np.array([1, 2, 3], dtype=np.int32)
    assert s.store_entry(_ctx(), toks, b"m" * 8, 1)
    # same key fields but a different model identity in the context
    e = s.entries()[0]
    assert e["entry_model_hash"] == 0x1111


def test_persistence_and_v8_and_reset(tmp_path):
    s = _store(tmp_path)
    toks = np.arange(10, dtype=np.int32)
    assert s.store_entry(_ctx(), toks, b"p" * 32, 3)
    s.shutdown()
    s2 = _store(tmp_path)
    assert s2.entry_count == 1
    r, e = s2.find_longest_prefix(_ctx(), toks)
    assert r == "hit" and s2.load_kv(e) == b"p" * 32
    s2.shutdown()
    # corrupt the checksum -> store disables (fail closed)
    p = os.path.join(tmp_path, "amf_index.bin")
    data = bytearray(open(p, "rb").read())
    data[30] ^= 0x55
    open(p, "wb").write(bytes(data))
    s3 = native().AmfStore()
    assert not s3.init(str(tmp_path), {"min_tokens": 2})
    assert s3.disabled_reason == "io_error"
    # a future version resets to a cold start instead of disabling
    hdr = struct.pack("<IIQQ", formats.INDEX_MAGIC, 99, 0, 0)
    open(p, "wb").write(hdr)
    s4 = native().AmfStore()
    assert s4.init(str(tmp_path), {"min_tokens": 2}) and s4.entry_count == 0
    # a v8 index (no tenant hash in the key) is readable
    rec = struct.pack("<QQIIIIQQ", 0x1111, 77, 4096, 0, 0, 0, 0x2222, 0x5555)
    body = rec + formats.RECORD_V9.pack(*([0] * 9 + [0x1111, 3, 0, 0, 0, float("nan"), float("nan"),
                                                      float("nan")] + [0] * 6 + [0, 0] + [0] * 7 + [1]))[56:]
    hdr0 = struct.pack("<IIQQ", formats.INDEX_MAGIC, 8, 1, 0)
    cs = native().fnv1a_bytes(hdr0 + body)
    open(p, "wb").write(struct.pack("<IIQQ", formats.INDEX_MAGIC, 8, 1, cs) + body)
    s5 = native().AmfStore()
    assert s5.init(str(tmp_path), {"min_tokens": 2}) and s5.entry_count == 1
    assert s5.entries()[0]["tenant_hash"] == 0 and s5.entries()[0]["prefix_hash"] == 77


def test_disk_guard_rejects(tmp_path):
    s = _store(tmp_path, min_free_disk_ratio=0.9999999)
    assert not s.store_entry(_ctx(), np.arange(4, dtype=np.int32), b"d" * 8, 1)
    assert s.stats()["admission_rejects"] == 1


def test_min_admit_roi_bootstrap_and_low_roi(tmp_path):
    s = _store(tmp_path, min_admit_roi=2.0, low_roi_hit_limit=2)
    c = _ctx()
    toks = np.arange(6, dtype=np.int32)
    assert s.store_entry(c, toks, b"r" * 8, 1)  # bootstrap admission
    r, e = s.find_longest_prefix(c, toks)
    s.note_hit(e, 6, 10, 1)   # restore 10 ms, saved 1 ms: roi 0.1
    s.note_hit(e, 6, 10, 1)   # second low-roi hit -> evicted
    assert s.entry_count == 0


def test_prewarm(tmp_path):
    s = _store(tmp_path)
    for i in range(3):
        assert s.store_entry(_ctx(), np.arange(i, i + 5, dtype=np.int32), bytes([i]) * 64, 1)
    s.shutdown()
    s2 = _store(tmp_path, prewarm=True, prewarm_top_k=2)
    for _ in range(200):
        if s2.prewarm_complete:
            break
        time.sleep(0.01)
    assert s2.prewarm_complete and s2.prewarm_loaded == 2 and s2.prewarm_failed == 0


def test_env_config(monkeypatch, tmp_path):
    monkeypatch.setenv("KORITH_ENABLE_AMF", "1")
    monkeypatch.setenv("KORITH_AMF_PATH", str(tmp_path))
    monkeypatch.setenv("KORITH_AMF_STORAGE_BUDGET_GB", "0.5")
    monkeypatch.setenv("KORITH_AMF_EVICTION_POLICY", "roi")
    monkeypatch.setenv("KORITH_AMF_HOT_TTL_S", "900")
    monkeypatch.setenv("KORITH_AMF_WARM_TTL_S", "60")
    d = native().store_config_from_env()
    assert d["enabled"] and d["path"] == str(tmp_path)
    assert d["storage_budget_bytes"] == 512 << 20 and d["policy"] == "roi"
    assert d["hot_ttl_ms"] == 60000  # hot TTL is clamped to the warm TTL
    monkeypatch.setenv("KORITH_ENABLE_AMF", "0")
    s = native().AmfStore()
    assert not s.init_from_env() and s.disabled_reason == "env_off"
