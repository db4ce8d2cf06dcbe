"""Numerics of every sm_100a kernel against the plain PyTorch fp32 oracle."""
import math

import pytest
import torch

from axropus_deploy_b200.amf.pool import DenseStore, PoolSlab
from axropus_deploy_b200.ops import (KVCache, argmax, decode_attention, page_transfer, prefill_attention, rmsnorm,
                                     rope_cos_sin, rope_kv_write, silu_mul, spec_verify)

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _fill_cache(c: KVCache, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    vals = torch.randn(c.num_blocks, c.num_layers, 2, c.num_kv_heads, 16, c.head_dim, generator=g)
    c.write_units(torch.arange(c.num_blocks), vals.to(c.device))
    return c


def _cpu_copy(c: KVCache) -> KVCache:
    d = KVCache(c.num_layers, c.num_blocks, c.num_kv_heads, c.head_dim, c.fmt_name, "cpu")
    d.data.copy_(c.data.cpu())
    if c.meta is not None:
        d.meta.copy_(c.meta.cpu())
    return d


@pytest.mark.parametrize("cache_fmt", ["bf16", "fp8", "int4"])
@pytest.mark.parametrize("pool_fmt", ["raw", "fp8", "int4"])
def test_page_transfer_roundtrip(cache_fmt, pool_fmt):
    L, NB, H, D = 2, 24, 4, 128
    cache = _fill_cache(KVCache(L, NB, H, D, cache_fmt, DEV), seed=1)
    slab = PoolSlab(32, L, H, D, pool_fmt, DEV)
    src = torch.tensor([3, 7, 1, 20, 5], dtype=torch.int32)
    slots = torch.tensor([9, 0, 31, 4, 17], dtype=torch.int32)
    page_transfer(cache, src, slab, slots)
    # oracle: same transfer on CPU copies
    cslab = PoolSlab(32, L, H, D, pool_fmt, "cpu")
    page_transfer(_cpu_copy(cache), src, cslab, slots)
    got = slab.read_units(slots.to(DEV)).cpu()
    want = cslab.read_units(slots)
    torch.testing.assert_close(got, want, atol=2e-2 * want.abs().max().item(), rtol=0)
    # restore into a fresh cache with a shuffled block table
    dst = KVCache(L, NB, H, D, cache_fmt, DEV)
    dblk = torch.tensor([11, 2, 19, 0, 6], dtype=torch.int32)
    page_transfer(slab, slots, dst, dblk)
    back = dst.read_units(dblk.to(DEV)).cpu()
    orig = cache.read_units(src.to(DEV)).cpu()
    if cache_fmt == "bf16" and pool_fmt == "raw":
        assert torch.equal(dst.data[:, :, dblk.long()].cpu(), cache.data[:, :, src.long()].cpu())  # bit exact
    tol = {"raw": 1e-2, "fp8": 0.08, "int4": 0.25}[pool_fmt] + (0.25 if cache_fmt == "int4" else 0.0)
    assert (back - orig).abs().max().item() <= tol * orig.abs().max().item()


def test_page_transfer_dense_roundtrip():
    L, H, D, n = 3, 2, 128, 5
    kv = torch.randn(L, 2, n * 16, H, D, device=DEV).to(torch.bfloat16)
    dense = DenseStore.from_tokens(kv)
    slab = PoolSlab(8, L, H, D, "raw", DEV)
    ids = torch.arange(n, dtype=torch.int32)
    page_transfer(dense, ids, slab, ids + 2)
    out = DenseStore(torch.empty_like(dense.t))
    page_transfer(slab, ids + 2, out, ids)
    assert torch.equal(out.to_tokens(), kv)


def _block_table(B, pages, NB, seed):
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(NB, generator=g)[: B * pages].view(B, pages)
    return perm.to(torch.int32)


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int4"])
@pytest.mark.parametrize("splits", [1, None])
def test_decode_attention(fmt, splits):
    L, H, D, G = 1, 2, 128, 4
    B, pages = 3, 9
    NB = B * pages + 4
    cache = _fill_cache(KVCache(L, NB, H, D, fmt, DEV), seed=2)
    bt = _block_table(B, pages, NB, 3)
    seq = torch.tensor([1, 77, 9 * 16], dtype=torch.int32)
    q = torch.randn(B, H * G, D).to(torch.bfloat16)
    out = decode_attention(q.to(DEV), cache, 0, bt.to(DEV), seq.to(DEV), num_splits=splits, max_seq_len=9 * 16)
    ref = decode_attention(q, _cpu_copy(cache), 0, bt, seq)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int4"])
def test_prefill_attention(fmt):
    L, H, D, G = 1, 2, 128, 4
    NB = 64
    cache = _fill_cache(KVCache(L, NB, H, D, fmt, DEV), seed=4)
    seq = torch.tensor([200, 70, 33], dtype=torch.int32)   # total cached tokens
    nq = torch.tensor([130, 70, 1], dtype=torch.int32)     # new tokens (suffix) of each
    cu = torch.zeros(4, dtype=torch.int32)
    cu[1:] = torch.cumsum(nq, 0)
    bt = _block_table(3, 13, NB, 5)
    q = torch.randn(int(cu[-1]), H * G, D).to(torch.bfloat16)
    out = prefill_attention(q.to(DEV), cache, 0, bt.to(DEV), cu.to(DEV), seq.to(DEV), int(nq.max()))
    ref = prefill_attention(q, _cpu_copy(cache), 0, bt, cu, seq, int(nq.max()))
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int4"])
@pytest.mark.parametrize("splits", [2, 5, 40])
def test_prefill_attention_split_kv(fmt, splits):
    """Suffix over a long cached prefix with the KV range split across CTAs (40 splits
    leaves some slices without keys for some query tiles)."""
    L, H, D, G = 1, 2, 128, 4
    NB = 214
    cache = _fill_cache(KVCache(L, NB, H, D, fmt, DEV), seed=6)
    seq = torch.tensor([1100, 700, 90], dtype=torch.int32)
    nq = torch.tensor([100, 3, 90], dtype=torch.int32)
    cu = torch.zeros(4, dtype=torch.int32)
    cu[1:] = torch.cumsum(nq, 0)
    bt = _block_table(3, 70, NB, 7)
    q = torch.randn(int(cu[-1]), H * G, D).to(torch.bfloat16)
    out = prefill_attention(q.to(DEV), cache, 0, bt.to(DEV), cu.to(DEV), seq.to(DEV), int(nq.max()),
                            num_splits=splits)
    ref = prefill_attention(q, _cpu_copy(cache), 0, bt, cu, seq, int(nq.max()))
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=3e-2, rtol=3e-2)
    auto = prefill_attention(q.to(DEV), cache, 0, bt.to(DEV), cu.to(DEV), seq.to(DEV), int(nq.max()),
                             max_seq_len=1100)
    torch.testing.assert_close(auto.cpu().float(), ref.float(), atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("pack", [True, False])
@pytest.mark.parametrize("G", [4, 8])
def test_prefill_attention_tcgen05_long(G, pack):
    """tcgen05 prefill kernel (bf16 pages) on multi-tile causal prefills and a suffix,
    with per-block key magnitudes from 1x to 8x so the running max moves by more than
    2^8 between KV tiles (the O rescale in TMEM runs); rows one head at a time, or the
    G query heads of a KV head packed into the same tiles."""
    from axropus_deploy_b200.ops import attention as att

    saved = att.GQA_PACK_MAX_Q[0]
    att.GQA_PACK_MAX_Q[0] = 2048 if pack else 0
    try:
        _tcgen05_long_case(G)
    finally:
        att.GQA_PACK_MAX_Q[0] = saved


def _tcgen05_long_case(G):
    from axropus_deploy_b200.ops import attention as att
    from axropus_deploy_b200.ops.gemm import check_errors

    L, H, D = 1, 2, 128
    seq = torch.tensor([700, 300, 129], dtype=torch.int32)
    nq = torch.tensor([700, 150, 129], dtype=torch.int32)
    pages = 45
    NB = 3 * pages + 5
    vals = torch.randn(NB, L, 2, H, 16, D, generator=torch.Generator().manual_seed(9))
    vals[:, :, 0] *= torch.linspace(1.0, 8.0, NB)[:, None, None, None, None]
    cache = KVCache(L, NB, H, D, "bf16", DEV)
    cache.write_units(torch.arange(NB), vals.to(DEV))
    cu = torch.zeros(4, dtype=torch.int32)
    cu[1:] = torch.cumsum(nq, 0)
    bt = _block_table(3, pages, NB, 11)
    q = (torch.randn(int(cu[-1]), H * G, D) * 2.0).to(torch.bfloat16)
    assert att.PREFILL_TC[0]
    out = prefill_attention(q.to(DEV), cache, 0, bt.to(DEV), cu.to(DEV), seq.to(DEV), int(nq.max()))
    torch.cuda.synchronize()
    assert check_errors(q.device if q.is_cuda else torch.device(DEV)) == 0
    ref = prefill_attention(q, _cpu_copy(cache), 0, bt, cu, seq, int(nq.max()))
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=3e-2, rtol=3e-2)
    att.PREFILL_TC[0] = False
    try:
        legacy = prefill_attention(q.to(DEV), cache, 0, bt.to(DEV), cu.to(DEV), seq.to(DEV), int(nq.max()))
    finally:
        att.PREFILL_TC[0] = True
    torch.testing.assert_close(out.float(), legacy.float(), atol=3e-2, rtol=3e-2)


@pytest.mark.parametrize("splits", [None, 1, 7])
def test_prefill_attention_tcgen05_packed_suffix(splits):
    """A 128-token suffix over a 4 K-token cached prefix (the AMF-hit shape), GQA-packed
    rows, with and without split KV, against the float32 reference."""
    L, H, D, G = 1, 8, 128, 4
    pages = 265
    NB = pages + 3
    cache = _fill_cache(KVCache(L, NB, H, D, "bf16", DEV), seed=12)
    seq = torch.tensor([4224], dtype=torch.int32)
    nq = torch.tensor([128], dtype=torch.int32)
    cu = torch.tensor([0, 128], dtype=torch.int32)
    bt = _block_table(1, pages, NB, 13)
    q = torch.randn(128, H * G, D).to(torch.bfloat16)
    out = prefill_attention(q.to(DEV), cache, 0, bt.to(DEV), cu.to(DEV), seq.to(DEV), 128, max_seq_len=4224,
                            num_splits=splits)
    ref = prefill_attention(q, _cpu_copy(cache), 0, bt, cu, seq, 128)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=3e-2, rtol=3e-2)


def test_rmsnorm_residual():
    x = torch.randn(37, 4096).to(torch.bfloat16)
    r = torch.randn(37, 4096).to(torch.bfloat16)
    w = (torch.rand(4096) + 0.5).to(torch.bfloat16)
    r_gpu = r.clone().to(DEV)
    out = rmsnorm(x.to(DEV), w.to(DEV), 1e-5, residual=r_gpu)
    r_ref = r.clone()
    ref = rmsnorm(x, w, 1e-5, residual=r_ref)
    torch.testing.assert_close(r_gpu.cpu(), r_ref)
    torch.testing.assert_close(out.cpu().float(), ref.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("fmt", ["bf16", "fp8", "int4"])
def test_rope_kv_write(fmt):
    Hq, Hkv, D, T = 8, 2, 128, 21
    cs = rope_cos_sin(4096, D, 500000.0, {"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                          "original_max_position_embeddings": 8192})
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D).to(torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), dtype=torch.int32)
    slots = torch.randperm(8 * 16)[:T].to(torch.int32)
    slots[3] = -1
    cg = KVCache(1, 8, Hkv, D, fmt, DEV)
    cc = KVCache(1, 8, Hkv, D, fmt, "cpu")
    qg = rope_kv_write(qkv.to(DEV), pos.to(DEV), slots.to(DEV), cs.to(DEV), cg, 0, Hq, Hkv)
    qc = rope_kv_write(qkv, pos, slots, cs, cc, 0, Hq, Hkv)
    torch.testing.assert_close(qg.cpu().float(), qc.float(), atol=1e-2, rtol=1e-2)
    ug = cg.read_units(torch.arange(8, device=DEV)).cpu()
    uc = cc.read_units(torch.arange(8))
    tol = {"bf16": 1e-2, "fp8": 0.1, "int4": 0.35}[fmt]
    assert (ug - uc).abs().max().item() <= tol


def test_silu_mul_argmax_verify():
    gu = torch.randn(9, 2 * 1024).to(torch.bfloat16)
    torch.testing.assert_close(silu_mul(gu.to(DEV)).cpu().float(), silu_mul(gu).float(), atol=2e-2, rtol=2e-2)
    logits = torch.randn(5, 128256)
    logits[2, 77] = 100.0
    assert torch.equal(argmax(logits.to(DEV)).cpu(), argmax(logits))
    lg = torch.randn(2, 5, 1000)
    draft = torch.argmax(lg[:, :4], -1).to(torch.int32)
    draft[1, 2] = (draft[1, 2] + 1) % 1000
    got = spec_verify(lg.to(DEV), draft.to(DEV)).cpu()
    assert torch.equal(got, spec_verify(lg, draft))
    assert got[0, 0].item() == 4 and got[1, 0].item() == 2
    # bf16 rows, ties (lowest index wins), rows not 16-byte aligned (V = 1001 bf16), tails
    for V in (128256, 1001, 37):
        lb = torch.randn(7, V).to(torch.bfloat16)
        lb[3, V // 3] = 50.0
        lb[3, V - 1] = 50.0
        lb[5] = 1.0
        assert torch.equal(argmax(lb.to(DEV)).cpu(), torch.argmax(lb.float(), -1).to(torch.int32)), V
    lgb = torch.randn(3, 9, 1001).to(torch.bfloat16)
    drb = torch.argmax(lgb[:, :8].float(), -1).to(torch.int32)
    drb[0, 5] = (drb[0, 5] + 1) % 1001
    gb = spec_verify(lgb.to(DEV), drb.to(DEV)).cpu()
    assert gb[:, 0].tolist() == [5, 8, 8] and torch.equal(gb, spec_verify(lgb.float(), drb))

