"""G1 pool (sharded directory + slabs) and the tiered router, on CPU."""
import pytest
import torch

from axropus_deploy_b200.amf import (CacheTier, G1Pool, LMCacheAdapter, MissReason, TieredCacheRouter, WritePolicy,
                                     compute_prefix_hash)
from axropus_deploy_b200.amf.keys import pool_key

L, H, D = 2, 4, 64


def _kv(T, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(L, 2, T, H, D, generator=g).to(torch.bfloat16)


@pytest.fixture
def pool():
    return G1Pool(L, H, D, "raw", slots_per_shard=16, device="cpu")


def test_insert_get_delete_roundtrip(pool):
    kv = _kv(64)
    assert pool.put_from_raw("aa11", kv)
    assert "aa11" in pool and len(pool) == 1
    e = pool.get("aa11")
    assert e.num_tokens == 64 and len(e.slots) == 4
    back = pool.restore_to_tensor("aa11")
    assert torch.equal(back, kv)  # raw pool is bit exact
    assert pool.delete("aa11") and "aa11" not in pool
    assert pool.get("aa11") is None


@pytest.mark.parametrize("fmt,tol", [("fp8", 0.07), ("int4", 0.12)])
def test_compressed_roundtrip(fmt, tol):
    p = G1Pool(L, H, D, fmt, slots_per_shard=8, device="cpu")
    kv = _kv(48, 1)
    assert p.put_from_raw("bb22", kv)
    back = p.restore_to_tensor("bb22").float()
    assert (back - kv.float()).abs().max() <= tol * kv.float().abs().max()
    assert p.used_bytes() == 3 * p.chunk


def test_eviction_under_pressure_and_pins(pool):
    for i in range(4):
        assert pool.put_from_raw(f"{i + 1:04x}", _kv(64, i))  # 4 x 4 slots = full
    hit = pool.lookup("0001")  # pinned
    assert pool.put_from_raw("00ff", _kv(64, 9))  # evicts someone, never the pinned one
    assert "0001" in pool and "00ff" in pool and len(pool) == 4
    assert pool.stats()["evictions"] == 1
    pool.release(hit)
    assert pool.put_from_raw("0a0a", _kv(256, 3)) is False or len(pool) >= 1  # 16 slots fits after evicting all


def test_reuse_score_protects_recent(pool):
    for i in range(4):
        assert pool.put_from_raw(f"{i + 1:04x}", _kv(64, i))
    for _ in range(5):
        pool.get("0004")
    assert pool.put_from_raw("0099", _kv(64, 7))
    assert "0004" in pool


def test_bad_shape_and_too_large(pool):
    with pytest.raises(ValueError):
        pool.put_from_raw("ab", torch.zeros(2, 3, 4))
    assert not pool.put_from_raw("cd", _kv(8))  # less than one page
    assert not pool.put_from_raw("ef", _kv(16 * 17))  # more pages than the shard has


def test_map_into_block_table(pool):
    assert pool.put_from_raw("1234", _kv(32))
    table = {7: []}
    assert pool.map_into_vllm("1234", 7, table)
    assert len(table[7]) == 2 and table[7][0]["is_external"]
    assert not pool.map_into_vllm("ffff", 7, table)


def test_router_tiers_and_miss_reasons(pool, tmp_path):
    lm = LMCacheAdapter(enabled=True, backend="cpu")
    r = TieredCacheRouter(pool, lm, min_prefix_tokens=16, write_policy=WritePolicy.ALWAYS)
    toks = list(range(64))
    h = compute_prefix_hash(toks)
    assert h == pool_key(toks) and len(h) == 16
    res = r.lookup(h, toks)
    assert res.tier == CacheTier.COLD and res.miss_reason == MissReason.FIRST_REQUEST
    assert r.store_after_prefill(h, toks, _kv(64))
    assert r.lookup(h, toks).tier == CacheTier.G1_AMF
    pool.delete(h)
    res = r.lookup(h, toks)  # G1 evicted, LMCache has it -> promoted back
    assert res.tier == CacheTier.G3_LMCACHE and h in pool
    assert r.lookup(h, toks[:8]).miss_reason == MissReason.PREFIX_TOO_SHORT
    lm.evict(h)
    pool.delete(h)
    assert r.lookup(h, toks).miss_reason == MissReason.EVICTED_FROM_AMF
    s = r.stats()
    assert s["tier_hits"]["amf"] == 1 and s["tier_hits"]["lmcache"] == 1 and s["write_policy"] == "always"


def test_router_write_policies(pool):
    r = TieredCacheRouter(pool, LMCacheAdapter(enabled=True), write_policy=WritePolicy.LARGE_ONLY,
                          large_write_threshold=2048)
    assert not r.should_mirror(100) and r.should_mirror(4096)
    r.write_policy = WritePolicy.NEVER
    assert not r.should_mirror(10 ** 6)
    r.write_policy = WritePolicy.ON_EVICTION
    assert not r.should_mirror(10 ** 6) and r.should_mirror(10, is_eviction=True)


def test_router_prefetch_resolver(pool):
    r = TieredCacheRouter(pool, LMCacheAdapter(enabled=False))
    kv = _kv(32, 5)
    r.set_prefetch_resolver(lambda key: kv if key == "beef" else None)
    r.prefetch("beef")
    import time

    for _ in range(100):
        if "beef" in pool:
            break
        time.sleep(0.02)
    r.stop_prefetch()
    assert "beef" in pool and torch.equal(pool.restore_to_tensor("beef"), kv)


def test_nvme_tier(tmp_path):
    lm = LMCacheAdapter(enabled=True, backend="nvme", path=str(tmp_path))
    pages = torch.randn(2, L, 2, H, 16, D).to(torch.bfloat16)
    assert lm.store("k1", pages) and lm.contains("k1")
    assert torch.equal(lm.lookup("k1"), pages)
    assert (tmp_path / "k1.pt").exists()


def test_cpu_tier_page_arena_runs_and_lru():
    """CPU tier on a pre-pinned page arena: entries are contiguous runs, LRU entries are
    evicted until a run fits, freed runs merge back."""
    from axropus_deploy_b200.amf.lmcache import LMCacheAdapter, PinnedPageArena

    shape = (2, 2, 1, 16, 8)
    page_bytes = 2 * 2 * 1 * 16 * 8 * 2
    lm = LMCacheAdapter(enabled=True, backend="cpu", max_bytes=10 * page_bytes)
    lm.reserve(shape)
    assert lm._arena is not None and lm._arena.n_pages == 10
    pages = {k: torch.full((n, *shape), float(i + 1)).to(torch.bfloat16) for i, (k, n) in
             enumerate([("a", 4), ("b", 3), ("c", 3)])}
    for k, v in pages.items():
        assert lm.store(k, v)
    assert lm._arena.free == []
    assert torch.equal(lm.lookup("b"), pages["b"])  # b becomes most recently used
    assert lm.store("d", torch.zeros(4, *shape, dtype=torch.bfloat16))  # evicts a (LRU) only
    assert lm.lookup("a") is None
    assert torch.equal(lm.lookup("b"), pages["b"]) and torch.equal(lm.lookup("c"), pages["c"])
    # LRU order is now d, b, c; 5 contiguous pages need d's run (0-3) and b's (4-6) merged
    assert lm.store("e", torch.zeros(5, *shape, dtype=torch.bfloat16))
    assert lm.lookup("d") is None and lm.lookup("b") is None
    assert torch.equal(lm.lookup("c"), pages["c"])
    assert lm.evict("e") and lm.evict("c")
    assert lm._arena.free == [(0, 10)]
    ar = PinnedPageArena(8, (1,))
    s1, s2 = ar.alloc(3), ar.alloc(3)
    ar.release(s1, 3)
    assert ar.alloc(4) is None and ar.alloc(3) == s1
