"""GPU codec kernels (csrc/kernels/codecs.cu) against the PyTorch codecs: the same bytes
(codes and scales) for fp32 / fp16 / bf16 inputs and odd shapes, decoding within the
reference tolerances, and blobs written on one side decoding on the other."""
import pytest
import torch

from axropus_deploy_b200 import codecs as C

pytestmark = pytest.mark.gpu

TOL = {"int4_sym": 0.20, "int4_sym_block": 0.22, "int2_sym": 0.70, "nvfp4": 0.15}
SHAPES = [(2, 256, 8, 128), (3, 300, 2, 33), (1, 129, 1, 16), (5, 7, 3, 9)]


def _launches():
    from axropus_deploy_b200.ops._ext import launches
    return launches()


@pytest.mark.parametrize("fmt", sorted(TOL))
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", SHAPES)
def test_gpu_codec_bytes_match_cpu(fmt, dtype, shape):
    torch.manual_seed(len(fmt) * 1000 + sum(shape))
    x = (torch.randn(*shape) * torch.rand(shape[-1]) * 3).to(dtype)
    codec = C.get_codec(fmt)
    cpu = codec.compress(x)
    n0 = _launches()
    gpu = codec.compress(x.cuda())
    assert _launches() > n0, "the CUDA codec did not run"
    assert gpu.data.is_cuda and gpu.data.shape == cpu.data.shape and gpu.scales.shape == cpu.scales.shape
    assert torch.equal(gpu.scales.cpu(), cpu.scales), fmt
    assert torch.equal(gpu.data.cpu(), cpu.data), fmt
    assert gpu.meta == cpu.meta
    if fmt == "nvfp4":
        assert gpu.tensor_scale == pytest.approx(cpu.tensor_scale, rel=1e-6)
    for out_dtype in (torch.float32, torch.bfloat16):
        got = codec.decompress_to(gpu, out_dtype)
        assert got.is_cuda and got.dtype == out_dtype and got.shape == x.shape
        want = codec.decompress_to(cpu, out_dtype)
        assert torch.equal(got.cpu(), want), (fmt, out_dtype)


@pytest.mark.parametrize("fmt", sorted(TOL))
def test_gpu_codec_reference_tolerance(fmt):
    torch.manual_seed(0)
    kv = torch.randn(2, 256, 8, 128, device="cuda")
    codec = C.get_codec(fmt)
    out = codec.decompress_to(codec.compress(kv), torch.float32)
    rel = ((out - kv).norm() / kv.norm()).item()
    assert rel < TOL[fmt], (fmt, rel)


def test_gpu_turboquant_runs_on_device():
    torch.manual_seed(0)
    kv = torch.randn(2, 64, 8, 128, device="cuda")
    c = C.get_codec("turboquant")
    blob = c.compress(kv)
    assert blob.data.is_cuda
    out = c.decompress_to(blob, torch.float32)
    assert ((out - kv).norm() / kv.norm()).item() < 0.60
