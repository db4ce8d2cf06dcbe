"""Small, self-contained cases of each hot kernel, for profiling one kernel at a time
(e.g. under ncu with -k/-c). Sizes are chosen so inputs exceed the 126 MB L2 while the
whole run stays within a few GB of device memory.

    python benchmarks/kernel_cases.py decode|decode_int4|decode_fp8|decode_shared|restore|restore_fp8|capture_int4|
                                      prefill|prefill_split|gemm|gemm_tp|moe|rmsnorm|rope|
                                      silu_mul|argmax|spec_verify
"""
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from axropus_deploy_b200 import ops  # noqa: E402
from axropus_deploy_b200.amf.pool import PoolSlab  # noqa: E402
from axropus_deploy_b200.ops import KVCache  # noqa: E402
from axropus_deploy_b200.ops.gemm import gemm  # noqa: E402


def decode(fmt="bf16"):
    # Llama-3-8B attention geometry: 32 q heads / 8 kv heads, batch 32, 4096-token context
    B, T = 32, 4096
    pages = T // 16
    cache = KVCache(1, B * pages, 8, 128, fmt, "cuda")
    if fmt == "bf16":
        cache.data.normal_()
    else:
        cache.data.random_(0, 255)
        cache.meta.fill_(0.01)
    bt = torch.randperm(B * pages, device="cuda").to(torch.int32).view(B, pages)
    sl = torch.full((B,), T, dtype=torch.int32, device="cuda")
    q = torch.randn(B, 32, 128, device="cuda").to(torch.bfloat16)
    for _ in range(3):
        ops.decode_attention(q, cache, 0, bt, sl, max_seq_len=T)


def decode_shared():
    # the headline bench's decode batch: 32 sequences of 8448 tokens whose 8192-token
    # prefixes follow its Zipf(1.1) reuse over 64 prefixes (10 % fresh), one layer
    import numpy as np

    from decode_step import build_tables

    class A:
        batch, context, prefix_len, prefixes = 32, 8448, 8192, 64

    lists, nblocks = build_tables(A, np.random.default_rng(0))
    cache = KVCache(1, nblocks + 8, 8, 128, "bf16", "cuda")
    cache.data.normal_()
    width = max(len(x) for x in lists)
    bt = torch.zeros(A.batch, width, dtype=torch.int32)
    for i, x in enumerate(lists):
        bt[i, :len(x)] = torch.tensor(x, dtype=torch.int32)
    bt = bt.cuda()
    sl = torch.full((A.batch,), A.context, dtype=torch.int32, device="cuda")
    q = torch.randn(A.batch, 32, 128, device="cuda").to(torch.bfloat16)
    for _ in range(3):
        ops.decode_attention(q, cache, 0, bt, sl, max_seq_len=A.context)


def restore(pool_fmt="raw", cache_fmt="bf16"):
    # one 8192-token prefix of a 32-layer / 8-kv-head model (1 GiB bf16): pool -> live cache
    slab = PoolSlab(512, 32, 8, 128, pool_fmt, "cuda")
    slab.slab.random_(0, 255)
    if pool_fmt == "fp8":
        for s in range(512):  # keep the per-page scales finite
            slab.slab[s * slab.chunk + slab.data_region: s * slab.chunk + slab.data_region + slab.n_units * 4].view(
                torch.float32).fill_(0.01)
    cache = KVCache(32, 600, 8, 128, cache_fmt, "cuda")
    src = torch.arange(512, dtype=torch.int32, device="cuda")
    dst = torch.randperm(600, device="cuda")[:512].to(torch.int32)
    for _ in range(3):
        ops.page_transfer(slab, src, cache, dst)


def capture(pool_fmt="int4"):
    cache = KVCache(32, 600, 8, 128, "bf16", "cuda")
    cache.data.normal_()
    slab = PoolSlab(512, 32, 8, 128, pool_fmt, "cuda")
    src = torch.randperm(600, device="cuda")[:512].to(torch.int32)
    dst = torch.arange(512, dtype=torch.int32, device="cuda")
    for _ in range(3):
        ops.page_transfer(cache, src, slab, dst)


def prefill():
    T = 4096
    cache = KVCache(1, T // 16, 8, 128, "bf16", "cuda")
    cache.data.normal_()
    bt = torch.arange(T // 16, dtype=torch.int32, device="cuda").view(1, -1)
    cu = torch.tensor([0, T], dtype=torch.int32, device="cuda")
    sl = torch.tensor([T], dtype=torch.int32, device="cuda")
    q = torch.randn(T, 32, 128, device="cuda").to(torch.bfloat16)
    for _ in range(3):
        ops.prefill_attention(q, cache, 0, bt, cu, sl, T)


def gemm_case():
    a = torch.randn(8192, 4096, device="cuda").to(torch.bfloat16)
    w = torch.randn(6144, 4096, device="cuda").to(torch.bfloat16)
    for _ in range(3):
        gemm(a, w)


def rmsnorm():
    x = torch.randn(32768, 4096, device="cuda").to(torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.ones(4096, device="cuda").to(torch.bfloat16)
    for _ in range(3):
        ops.rmsnorm(x, w, 1e-5, residual=r)


def rope():
    T = 32768
    qkv = torch.randn(T, 6144, device="cuda").to(torch.bfloat16)
    cache = KVCache(1, T // 16, 8, 128, "bf16", "cuda")
    pos = torch.arange(T, dtype=torch.int32, device="cuda")
    cs = ops.rope_cos_sin(T, 128, 500000.0, None, "cuda")
    for _ in range(3):
        ops.rope_kv_write(qkv, pos, pos.clone(), cs, cache, 0, 32, 8)


def prefill_split():
    # 128-token suffix over an 8192-token cached prefix (hit TTFT case): split-KV prefill
    T, n = 8320, 128
    cache = KVCache(1, T // 16 + 1, 8, 128, "bf16", "cuda")
    cache.data.normal_()
    bt = torch.arange(T // 16 + 1, dtype=torch.int32, device="cuda").view(1, -1)
    cu = torch.tensor([0, n], dtype=torch.int32, device="cuda")
    sl = torch.tensor([T], dtype=torch.int32, device="cuda")
    q = torch.randn(n, 32, 128, device="cuda").to(torch.bfloat16)
    for _ in range(3):
        ops.prefill_attention(q, cache, 0, bt, cu, sl, n, max_seq_len=T)


def gemm_tp_plain():
    from axropus_deploy_b200.parallel.tp import TpGemm

    a = torch.randn(8192, 8192, device="cuda").to(torch.bfloat16)
    w = torch.randn(7168, 8192, device="cuda").to(torch.bfloat16)
    for _ in range(3):
        TpGemm.gemm(a, w)


def moe():
    # one Mixtral MoE layer, all 8 experts on this GPU (expert-parallel group of one), 4096 tokens
    from axropus_deploy_b200.parallel.dist import DistInfo
    from axropus_deploy_b200.parallel.ep import EpMoE, route

    E, H, F, T = 8, 4096, 14336, 4096
    dev = torch.device("cuda", 0)
    m = EpMoE(DistInfo(0, 1, 0, 1, dev), E, H, F, 2, max_tokens=T)
    w13 = (torch.randn(E, 2 * F, H, device=dev) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, H, F, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, H, device=dev).to(torch.bfloat16)
    idx, w = route(torch.randn(T, E, device=dev), 2)
    for _ in range(3):
        m.forward(x, idx, w, w13, w2)


def silu_mul():
    # Llama-3-8B MLP of an 8K-token prefill: gate|up [8192, 2 x 14336] -> [8192, 14336]
    gu = torch.randn(8192, 2 * 14336, device="cuda").to(torch.bfloat16)
    out = torch.empty(8192, 14336, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        ops.silu_mul(gu, out)


def argmax():
    # greedy sampling over the Llama-3 vocabulary, 1024 rows (263 MB of bf16 logits)
    logits = torch.randn(1024, 128256, device="cuda").to(torch.bfloat16)
    out = torch.empty(1024, dtype=torch.int32, device="cuda")
    for _ in range(3):
        ops.argmax(logits, out)


def spec_verify():
    # speculative verification: 64 sequences x (8 drafted + 1) positions over the vocabulary
    logits = torch.randn(64, 9, 128256, device="cuda").to(torch.bfloat16)
    draft = torch.randint(0, 128256, (64, 8), device="cuda", dtype=torch.int32)
    for _ in range(3):
        ops.spec_verify(logits, draft)


CASES = {"decode": lambda: decode("bf16"), "decode_int4": lambda: decode("int4"),
         "decode_fp8": lambda: decode("fp8"), "decode_shared": decode_shared,
         "restore": lambda: restore("raw", "bf16"),
         "restore_fp8": lambda: restore("fp8", "bf16"), "capture_int4": lambda: capture("int4"),
         "prefill": prefill, "gemm": gemm_case, "rmsnorm": rmsnorm, "rope": rope,
         "prefill_split": prefill_split, "gemm_tp": gemm_tp_plain, "moe": moe, "silu_mul": silu_mul,
         "argmax": argmax, "spec_verify": spec_verify}

if __name__ == "__main__":
    for name in sys.argv[1:] or ["decode"]:
        CASES[name]()
    torch.cuda.synchronize()
    print("ok", *sys.argv[1:])
