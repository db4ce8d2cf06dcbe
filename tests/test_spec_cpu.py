"""Speculative decoding (draft -> device verify -> roll back) must emit exactly the
greedy tokens of plain decoding; the n-gram drafter must find repeats."""
import torch

from axropus_deploy_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
from axropus_deploy_b200.engine.spec import NgramDrafter
from axropus_deploy_b200.models.config import get_config
from axropus_deploy_b200.models.llama import LlamaModel


def test_ngram_drafter():
    d = NgramDrafter()
    assert d.propose([1, 2, 3, 9, 9, 1, 2, 3], 3) == [9, 9, 1]
    assert d.propose([5, 6, 7, 5], 2) == [6, 7]          # 1-gram fallback
    assert d.propose([4], 2) == [4, 4]


def _model():
    return LlamaModel(get_config("tiny128"), "cpu", torch.float32, seed=7, init_std=0.05)


def _prompts():
    g = torch.Generator().manual_seed(2)
    base = torch.randint(0, 32000, (40,), generator=g).tolist()
    return [base * 3, torch.randint(0, 32000, (70,), generator=g).tolist()]


def test_spec_ngram_matches_greedy():
    m = _model()
    ref = LLMEngine(m, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512)).generate(
        _prompts(), SamplingParams(max_tokens=24))
    eng = LLMEngine(m, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512, spec="ngram"))
    got = eng.generate(_prompts(), SamplingParams(max_tokens=24))
    assert got == ref
    st = eng.stats()["spec"]
    assert st["steps"] > 0 and st["emitted"] >= st["seq_steps"]


def test_spec_draft_model_matches_greedy():
    m = _model()
    ref = LLMEngine(m, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512)).generate(
        _prompts(), SamplingParams(max_tokens=12))
    # the target as its own draft model: every draft is accepted
    eng = LLMEngine(m, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512, spec="model"), draft_model=m)
    got = eng.generate(_prompts(), SamplingParams(max_tokens=12))
    assert got == ref
    st = eng.stats()["spec"]
    assert st["acceptance"] > 0.9
