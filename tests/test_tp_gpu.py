"""Fused tensor-parallel GEMM kernels (csrc/kernels/gemm_tp.cu) against float32 references.

One GPU: the persistent kernel without communication, and the all-gather / reduce-scatter
modes with a group of one (flags, staging and receive paths run; nothing crosses NVLink).
Two or more GPUs: ``benchmarks/tp_gemm.py --check-only --small`` under torchrun, one rank
per GPU, peers exchanging rows and partial tiles over NVLink.
"""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rel(x, ref):
    return float((x.float() - ref).norm() / ref.norm())


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1000, 1280, 8192), (4096, 4096, 1024), (300, 200, 96)])
def test_gemm_tp_plain(M, N, K):
    from axropus_deploy_b200.ops.gemm import check_errors
    from axropus_deploy_b200.parallel.tp import TpGemm

    torch.manual_seed(0)
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * K ** -0.5).to(torch.bfloat16)
    for _ in range(2):  # second call: accumulators and barriers reused
        y = TpGemm.gemm(a, w)
    torch.cuda.synchronize()
    assert check_errors(a.device) == 0
    assert _rel(y, a.float() @ w.float().t()) < 1e-2


@pytest.mark.gpu
def test_gemm_tp_group_of_one():
    from axropus_deploy_b200.ops.gemm import check_errors
    from axropus_deploy_b200.parallel.dist import DistInfo
    from axropus_deploy_b200.parallel.tp import TpGemm

    info = DistInfo(0, 1, 0, 1, torch.device("cuda", 0))
    tp = TpGemm(info, 512, 1024, 768)
    torch.manual_seed(1)
    for rows in (512, 256, 512):  # row counts may change between calls
        x = torch.randn(rows, 1024, device="cuda").to(torch.bfloat16)
        w = (torch.randn(640, 1024, device="cuda") * 0.03).to(torch.bfloat16)
        y = tp.ag_gemm(x, w)
        a = torch.randn(rows, 512, device="cuda").to(torch.bfloat16)
        w2 = (torch.randn(768, 512, device="cuda") * 0.04).to(torch.bfloat16)
        z = tp.gemm_rs(a, w2)
        torch.cuda.synchronize()
        assert check_errors(x.device) == 0
        assert _rel(y, x.float() @ w.float().t()) < 1e-2
        assert _rel(z, a.float() @ w2.float().t()) < 1e-2


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_gemm_tp_two_gpus():
    n = 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", "29531",
           os.path.join(ROOT, "benchmarks", "tp_gemm.py"), "--check-only", "--small"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_CHECK ok" in r.stdout


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_llama_two_gpus():
    """Tensor-parallel Llama (fused sequence-parallel prefill, replicated decode) vs the dense model."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29532",
           os.path.join(ROOT, "benchmarks", "tp_llama.py"), "--check"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_LLAMA_CHECK ok" in r.stdout


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_allreduce_two_gpus():
    """One-shot peer all-reduce vs NCCL, repeated and from a captured CUDA graph."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29535",
           os.path.join(ROOT, "benchmarks", "allreduce.py"), "--check"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "AR_CHECK ok" in r.stdout
