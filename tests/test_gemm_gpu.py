"""tcgen05 GEMM numerics against the fp32 PyTorch oracle."""
import pytest
import torch

from axropus_deploy_b200.ops.gemm import check_errors, gemm

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (1000, 768, 4096), (77, 300, 136),
                                   (4096, 6144, 4096)])
def test_gemm_tc(M, N, K):
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16).cuda()
    out = gemm(a, w)
    torch.cuda.synchronize()
    assert check_errors(a.device) == 0
    ref = a.float() @ w.float().t()
    err = (out.float() - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-2, err


def test_gemm_tc_residual_alpha():
    a = torch.randn(300, 512).to(torch.bfloat16).cuda()
    w = (torch.randn(512, 512) / 22.6).to(torch.bfloat16).cuda()
    r = torch.randn(300, 512).to(torch.bfloat16).cuda()
    out = gemm(a, w, residual=r, alpha=0.5)
    ref = 0.5 * (a.float() @ w.float().t()) + r.float()
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=2e-2)
