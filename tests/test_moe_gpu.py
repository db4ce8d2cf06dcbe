"""Fused MoE kernels (csrc/kernels/moe.cu) against the float32 expert reference.

One GPU: the dispatch / grouped GEMM / combine path with an expert-parallel group of one
(all experts local). Two GPUs: ``benchmarks/ep_moe.py --check`` under torchrun."""
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
@pytest.mark.parametrize("T", [0, 1, 300, 2000])
def test_moe_single_gpu(T):
    from axropus_deploy_b200.ops.gemm import check_errors
    from axropus_deploy_b200.parallel.dist import DistInfo
    from axropus_deploy_b200.parallel.ep import EpMoE, experts_reference, route

    dev = torch.device("cuda", 0)
    E, H, F, K = 4, 512, 768, 2
    moe = EpMoE(DistInfo(0, 1, 0, 1, dev), E, H, F, K, max_tokens=2048)
    g = torch.Generator(device=dev).manual_seed(T)
    w13 = (torch.randn(E, 2 * F, H, generator=g, device=dev) * 0.03).to(torch.bfloat16)
    w2 = (torch.randn(E, H, F, generator=g, device=dev) * 0.03).to(torch.bfloat16)
    for it in range(2):
        x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
        idx, w = route(torch.randn(T, E, generator=g, device=dev), K)
        y = moe.forward(x, idx, w, w13, w2)
        torch.cuda.synchronize()
        assert check_errors(dev) == 0
        if T:
            ref = experts_reference(x, idx, w, w13, w2)
            assert float((y.float() - ref).norm() / ref.norm()) < 2e-2


@pytest.mark.gpu
def test_moe_model_single_gpu():
    """tiny-moe model prefill on the fused MoE path vs the reference expert loop (logits)."""
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import AttnMeta, LlamaModel
    from axropus_deploy_b200.ops.kvcache import KVCache

    cfg = get_config("tiny-moe")
    m = LlamaModel(cfg, "cuda", seed=1, init_std=0.05)
    assert m.ep is not None
    T = 300
    dev = torch.device("cuda", 0)
    tokens = torch.arange(5, 5 + T, dtype=torch.int32, device=dev)
    pos = torch.arange(T, dtype=torch.int32, device=dev)
    bt = torch.arange(32, dtype=torch.int32, device=dev)[None]
    outs = []
    for use_ep in (True, False):
        ep = m.ep
        if not use_ep:
            m.ep = None
        cache = KVCache(m.num_layers, 32, cfg.num_kv_heads, cfg.head_dim, "bf16", dev)
        meta = AttnMeta("prefill", pos, pos, bt, torch.tensor([T], dtype=torch.int32, device=dev),
                        cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), max_q=T, max_seq_len=T,
                        logits_idx=torch.tensor([T - 1, 100], dtype=torch.int32, device=dev))
        outs.append(m.forward(tokens, meta, cache))
        m.ep = ep
    assert float((outs[0] - outs[1]).norm() / outs[1].norm()) < 3e-2


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_moe_two_gpus():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", "29541",
           os.path.join(ROOT, "benchmarks", "ep_moe.py"), "--check"]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "EP_CHECK ok" in r.stdout
