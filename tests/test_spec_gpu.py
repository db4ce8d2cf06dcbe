"""Speculative decoding on the GPU: the verify forward runs the prefill kernels, plain
decoding the decode kernels, so bf16 rounding may flip a near-tie; nearly all tokens must
agree and the draft model run (target as its own draft) must accept almost everything."""
import pytest
import torch


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
    ref = LLMEngine(m, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512)).generate(prompts, sp)
    for mode, kw in (("ngram", {}), ("model", {"draft_model": m})):
        eng = LLMEngine(m, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512, spec=mode), **kw)
        got = eng.generate(prompts, sp)
        agree = sum(a == b for x, y in zip(got, ref) for a, b in zip(x, y)) / sum(len(x) for x in ref)
        assert agree > 0.9, (mode, agree)
        if mode == "model":
            assert eng.stats()["spec"]["acceptance"] > 0.8
