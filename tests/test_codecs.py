"""Codecs: reference tolerances on randn(2,256,8,128) seed 0, packing conventions,
page formats, FP8 sidecar, and interop with the reference's own codecs when the
reference package is installed next to the repo (baseline/_ref)."""
import os
import sys

import pytest
import torch

from axropus_deploy_b200 import codecs as C

TOL = {"fp8_e4m3": 0.05, "fp8_e5m2": 0.10, "int4_sym": 0.20, "int4_sym_block": 0.22, "int2_sym": 0.70,
       "nvfp4": 0.15, "turboquant": 0.60, "fp8_e4m3_block": 0.05, "int4_g64_asym": 0.12}


@pytest.fixture(scope="module")
def kv():
    torch.manual_seed(0)
    return torch.randn(2, 256, 8, 128)


@pytest.mark.parametrize("fmt", sorted(TOL))
def test_roundtrip_tolerance(kv, fmt):
    c = C.get_codec(fmt)
    blob = c.compress(kv)
    out = c.decompress_to(blob, torch.float32)
    assert out.shape == kv.shape
    rel = ((out - kv).norm() / kv.norm()).item()
    assert rel < TOL[fmt], (fmt, rel)
    assert blob.nbytes() <= kv.numel() * 2 * (c.memory_ratio() + 0.02)


def test_registry_and_selector():
    assert set(TOL) <= set(C.list_codecs())
    with pytest.raises(KeyError):
        C.get_codec("nope")
    assert C.select_codec(100) == C.FMT_NVFP4
    assert C.select_codec(100, density_budget=0.2) == C.FMT_TURBOQUANT
    assert C.select_codec(90) == C.FMT_INT4_BLOCK and C.select_codec(90, density_budget=0.5) == C.FMT_FP8_E4M3
    assert C.select_codec(80) == C.FMT_INT4_BLOCK and C.select_codec(70) == C.FMT_FP16


def test_packing_conventions():
    q = torch.tensor([[-8, 7, 0, -1, 3]], dtype=torch.int8)
    p = C.pack_int4(q)
    assert p.tolist() == [[(0) | (15 << 4), (8) | (7 << 4), 11]]
    assert C.unpack_int4(p, 5).tolist() == q.tolist()
    u = torch.tensor([[0, 1, 2, 3, 3]], dtype=torch.uint8)
    assert C.pack_int2(u).tolist() == [[0 | 1 << 2 | 2 << 4 | 3 << 6, 3]]
    assert C.unpack_int2(C.pack_int2(u), 5).tolist() == u.tolist()


def test_page_formats():
    x = torch.randn(3, 16, 128)
    q, s = C.quantize_fp8_page(x)
    assert q.dtype == torch.uint8 and s.shape == (3,)
    assert (C.dequantize_fp8_page(q, s) - x).abs().max() <= 0.07 * x.abs().max()
    p, m = C.quantize_int4_g64(x)
    assert p.shape == (3, 16, 64) and m.shape == (3, 16, 2, 2) and m.dtype == torch.float16
    y = C.dequantize_int4_g64(p, m)
    rng = (x.unflatten(-1, (2, 64)).amax(-1) - x.unflatten(-1, (2, 64)).amin(-1)).max()
    assert (y - x).abs().max() <= rng / 15 * 0.51 + 1e-3
    z = torch.zeros(1, 16, 128)
    assert C.dequantize_fp8_page(*C.quantize_fp8_page(z)).abs().max() == 0


def test_fp8_sidecar_and_apply():
    sc = C.FP8ScaleSidecar(0.5, 0.25)
    assert C.FP8ScaleSidecar.from_tensor(sc.to_tensor()) == sc

    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.register_buffer("_k_scale", torch.tensor(1.0))
            self._v_scale = 1.0
            self.calculate_kv_scales = True

    m = torch.nn.Sequential(Attn(), torch.nn.Linear(2, 2))
    n = C.apply_fp8_scales(m, sc)
    assert n == 2 and float(m[0]._k_scale) == 0.5 and m[0]._v_scale == 0.25
    assert m[0].calculate_kv_scales is False


REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "korith_vllm_ext")), reason="reference not installed")
@pytest.mark.parametrize("fmt", ["fp8_e4m3", "int4_sym", "int4_sym_block", "int2_sym", "nvfp4", "turboquant"])
def test_reference_interop(kv, fmt):
    sys.path.insert(0, REF)
    try:
        from korith_vllm_ext.codecs import get_codec as ref_get
    finally:
        sys.path.remove(REF)
    ours, theirs = C.get_codec(fmt), ref_get(fmt)
    x = kv[:, :64]
    # their blob decoded by us, our blob decoded by them: same values as the writer's own decode
    tb = theirs.compress(x)
    ob = ours.compress(x)
    for blob, wdec in ((tb, theirs), (ob, ours)):
        a = ours.decompress_to(blob, torch.float32)
        b = theirs.decompress_to(blob, torch.float32)
        assert torch.allclose(a, b, atol=1e-4, rtol=1e-3), fmt
    if fmt not in ("turboquant",):
        assert torch.equal(tb.data.view(torch.uint8), ob.data.view(torch.uint8)), fmt
