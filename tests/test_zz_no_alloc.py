"""GPU test of the allocation-free decode entry point, called through its exported
C symbol ``axr_decode_attention_noalloc`` (ctypes; declared in
csrc/kernels/decode_attn_noalloc.h), for callers that cannot allocate device memory at
call time. Its output must match the regular decode_attention entry point (which uses a
caller-provided scratch buffer) and the fp32 CPU oracle, on two calls in a row. This
file is named to be collected last."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from axropus_deploy_b200.ops._ext import ext_path

    lib = ctypes.CDLL(ext_path())
    fn = lib.axr_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong,
                   ctypes.c_longlong, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.axr_decode_noalloc_last_error.restype = ctypes.c_char_p
    lib.axr_decode_noalloc_scratch_floats.restype = ctypes.c_longlong
    return lib


def _case(seed, B, Hkv, G, pages, seq):
    from axropus_deploy_b200.ops import KVCache

    g = torch.Generator().manual_seed(seed)
    NB = B * pages + 3
    cache = KVCache(1, NB, Hkv, 128, "bf16", "cuda")
    cache.data.copy_(torch.randn(cache.data.shape, generator=g).to(torch.bfloat16))
    bt = torch.randperm(NB, generator=g)[: B * pages].view(B, pages).to(torch.int32).cuda()
    q = torch.randn(B, Hkv * G, 128, generator=g).to(torch.bfloat16).cuda()
    return cache, bt, torch.tensor(seq, dtype=torch.int32).cuda(), q


def _noalloc(lib, cache, bt, sl, q, splits, max_pages):
    k, v, _, _, bs, hs, _, _ = cache.layer_args(0)
    out = torch.empty_like(q)
    B, Hq, D = q.shape
    rc = lib.axr_decode_attention_noalloc(q.data_ptr(), out.data_ptr(), k, v, bs, hs, bt.data_ptr(), bt.stride(0),
                                          sl.data_ptr(), B, Hq, cache.num_kv_heads, D, 1.0 / D ** 0.5, splits,
                                          max_pages, torch.cuda.current_stream().cuda_stream)
    return rc, out


def _oracle(cache, bt, sl, q):
    """fp32 CPU reference of the same attention (the ops' PyTorch path on CPU tensors)."""
    from axropus_deploy_b200.ops import KVCache, decode_attention

    c = KVCache(1, cache.num_blocks, cache.num_kv_heads, 128, "bf16", "cpu")
    c.data.copy_(cache.data.cpu())
    return decode_attention(q.cpu(), c, 0, bt.cpu(), sl.cpu())


def test_noalloc_matches_decode_attention_two_calls():
    from axropus_deploy_b200.ops import decode_attention

    lib = _lib()
    # the last case: every sequence fills its table row exactly (seq_len == max_pages * 16)
    # and 4 splits do not divide the 9 pages
    cases = [(11, 3, 2, 4, 9, [1, 77, 144], (3, 1)), (12, 4, 2, 4, 6, [96, 5, 33, 90], (3, 1)),
             (14, 2, 2, 4, 9, [144, 144], (4, 2))]
    for seed, B, Hkv, G, pages, seq, split_list in cases:
        cache, bt, sl, q = _case(seed, B, Hkv, G, pages, seq)
        ref = _oracle(cache, bt, sl, q)
        for splits in split_list:
            rc, got = _noalloc(lib, cache, bt, sl, q, splits, pages)
            assert rc == 0, lib.axr_decode_noalloc_last_error()
            want = decode_attention(q, cache, 0, bt, sl, num_splits=splits, max_seq_len=pages * 16)
            torch.cuda.synchronize()
            torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=2e-2)
            torch.testing.assert_close(got.float().cpu(), ref.float(), atol=2e-2, rtol=2e-2)


def test_noalloc_rejects_table_overrun():
    lib = _lib()
    cache, bt, sl, q = _case(15, 2, 2, 4, 4, [60, 64])
    rc, _ = _noalloc(lib, cache, bt, sl, q, 2, 5)  # max_pages beyond the table row (bt_stride 4)
    assert rc == 3 and b"invalid" in lib.axr_decode_noalloc_last_error()


def test_noalloc_rejects_oversize():
    lib = _lib()
    cache, bt, sl, q = _case(13, 2, 2, 4, 4, [60, 64])
    cap = lib.axr_decode_noalloc_scratch_floats()
    splits = int(cap // (2 * 8 * 129)) + 1  # one split more than fits
    rc, _ = _noalloc(lib, cache, bt, sl, q, splits, 4)
    assert rc == 1
    assert b"scratch" in lib.axr_decode_noalloc_last_error()
