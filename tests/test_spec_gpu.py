"""Speculative decoding on the GPU. The verify forward runs the prefill kernels and plain
decoding the decode kernels, so bf16 rounding can flip a near-tie and the two token
streams may part ways; what must hold is that every emitted token is a greedy choice of
the target: its logit (from one prefill over prompt + output) is within rounding of the
row's maximum."""
import pytest
import torch


def _check_greedy(m, prompt, out, tol=0.08):
    from axropus_deploy_b200.models.llama import AttnMeta
    from axropus_deploy_b200.ops.kvcache import KVCache

    dev = m.device
    full = prompt + out
    T = len(full)
    nb = (T + 15) // 16 + 1
    cache = KVCache(m.num_layers, nb, m.cfg.num_kv_heads, m.cfg.head_dim, "bf16", dev)
    pos = torch.arange(T, dtype=torch.int32, device=dev)
    idx = torch.arange(len(prompt) - 1, T - 1, dtype=torch.int32, device=dev)
    meta = AttnMeta("prefill", pos, pos, torch.arange(nb, dtype=torch.int32, device=dev)[None],
                    torch.tensor([T], dtype=torch.int32, device=dev),
                    cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), max_q=T, max_seq_len=T, logits_idx=idx)
    logits = m.forward(torch.tensor(full, dtype=torch.int32, device=dev), meta, cache).float()
    best = logits.max(dim=1).values
    got = logits[torch.arange(len(out), device=dev), torch.tensor(out, device=dev)]
    return bool((got >= best - tol * (1 + best.abs())).all())


@pytest.mark.gpu
def test_spec_gpu_ngram_and_model():
    from axropus_deploy_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel

    m = LlamaModel(get_config("tiny128"), "cuda", seed=7, init_std=0.05)
    g = torch.Generator().manual_seed(2)
    base = torch.randint(0, 32000, (40,), generator=g).tolist()
    prompts = [base * 3, torch.randint(0, 32000, (70,), generator=g).tolist()]
    sp = SamplingParams(max_tokens=32)
    for mode, kw in (("ngram", {}), ("model", {"draft_model": m})):
        eng = LLMEngine(m, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512, spec=mode), **kw)
        got = eng.generate(prompts, sp)
        for p, o in zip(prompts, got):
            assert len(o) == 32
            assert _check_greedy(m, p, o), mode
        st = eng.stats()["spec"]
        assert st["steps"] > 0
        if mode == "model":
            assert st["acceptance"] > 0.8


@pytest.mark.gpu
def test_spec_gpu_pool_branches():
    """Pool of drafters on the GPU: an always-wrong drafter and the target as its own draft
    model; the second proposal is verified on a copy-on-write branch and wins, its pages
    are swapped in, and every emitted token is a greedy choice of the target."""
    from axropus_deploy_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
    from axropus_deploy_b200.engine.pool import DraftPool, PoolSpecDecoder
    from axropus_deploy_b200.engine.spec import ModelDrafter
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel

    class Wrong:
        def propose(self, tokens, k):
            return [(int(tokens[-1]) + 1) % 32000] * k

    m = LlamaModel(get_config("tiny128"), "cuda", seed=7, init_std=0.05)
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (61, 100)]
    eng = LLMEngine(m, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512))
    eng.spec = PoolSpecDecoder(eng, 6, DraftPool([Wrong(), ModelDrafter(m, 128)]))
    got = eng.generate(prompts, SamplingParams(max_tokens=32))
    for p, o in zip(prompts, got):
        assert len(o) == 32
        assert _check_greedy(m, p, o)
    st = eng.spec.stats()
    assert st["branch_wins"] > 0 and st["acceptance"] > 0.5
    eng.close()
