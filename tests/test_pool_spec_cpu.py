"""Pool of draft engines with copy-on-write KV branches (engine/pool.py), on CPU:
a forked branch shares the sequence's full pages, owns a copy of the partial page it
writes into, and writing it leaves the sequence's pages untouched; multi-draft speculative
decoding emits exactly the tokens of plain greedy decoding, verifies several branches per
step and keeps non-primary branches when they accept more (their pages swapped in)."""
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from axropus_deploy_b200.engine import EngineConfig, LLMEngine, SamplingParams  # noqa: E402
from axropus_deploy_b200.engine.pool import DraftPool, PoolSpecDecoder, fork_kv  # noqa: E402
from axropus_deploy_b200.engine.spec import ModelDrafter, NgramDrafter  # noqa: E402
from axropus_deploy_b200.models.config import get_config  # noqa: E402
from axropus_deploy_b200.models.llama import LlamaModel  # noqa: E402


def _model():
    return LlamaModel(get_config("tiny"), "cpu", seed=0)


def test_fork_is_copy_on_write():
    model = _model()
    eng = LLMEngine(model, EngineConfig(num_blocks=64, max_model_len=512))
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, model.cfg.vocab, (37,), generator=g).tolist()
    r = eng.add_request(prompt, SamplingParams(max_tokens=4))
    eng.step()  # prefill: KV of the prompt is in the cache
    L = r.seq_len
    view = fork_kv(eng, r, L - 1, L + 5)
    p0 = (L - 1) // 16
    assert view.blocks[:p0] == r.blocks[:p0]  # shared full pages
    assert view.private[0] not in r.blocks
    before = eng.cache.data[:, :, r.blocks[p0]].clone()
    assert torch.equal(eng.cache.data[:, :, view.private[0]], before)  # the partial page copied
    eng.cache.data[:, :, view.private[0]].fill_(7)  # the branch writes ...
    assert torch.equal(eng.cache.data[:, :, r.blocks[p0]], before)  # ... the sequence does not see it
    free = eng.bm.num_free()
    view.release(eng.bm)
    assert eng.bm.num_free() == free + len(view.blocks) - p0


def _run(model, spec, prompts, n_out):
    eng = LLMEngine(model, EngineConfig(num_blocks=256, max_model_len=1024, spec=spec, spec_max_depth=6))
    reqs = [eng.add_request(p, SamplingParams(max_tokens=n_out)) for p in prompts]
    while eng.has_unfinished():
        eng.step()
    eng.close()
    return [r.output for r in reqs], eng


def test_pool_speculation_is_lossless_and_uses_branches():
    model = _model()
    g = torch.Generator().manual_seed(2)
    base = torch.randint(0, model.cfg.vocab, (24,), generator=g).tolist()
    a, b, c = torch.randint(0, model.cfg.vocab, (3, 12), generator=g).tolist()
    tail = a[:3]
    # repetitive prompts (drafts get accepted), one whose tail occurred twice with different
    # continuations (the most-recent and the earlier-occurrence drafters disagree) and a random one
    prompts = [base * 4, tail + b + tail + c + tail, (base[:10] * 7)[:65],
               torch.randint(0, model.cfg.vocab, (50,), generator=g).tolist()]
    ref, _ = _run(model, "", prompts, 24)
    out, eng = _run(model, "pool", prompts, 24)
    assert out == ref
    st = eng.spec.stats()
    assert st["steps"] > 0
    assert sum(e["branches"] for e in st["engines"]) == st["branches"]

    class Other:  # always a second, different proposal: two branches per sequence and step
        def propose(self, tokens, k):
            return [(int(tokens[-1]) * 7 + i) % 1000 for i in range(k)]

    eng = LLMEngine(model, EngineConfig(num_blocks=256, max_model_len=1024))
    eng.spec = PoolSpecDecoder(eng, 6, DraftPool([NgramDrafter(3, 1), Other()]))
    reqs = [eng.add_request(p, SamplingParams(max_tokens=24)) for p in prompts]
    while eng.has_unfinished():
        eng.step()
    assert [r.output for r in reqs] == ref
    st = eng.spec.stats()
    assert st["branches"] > st["seq_steps"]  # several proposals verified per sequence and step


def test_pool_keeps_a_better_second_branch():
    """A pool whose first drafter always proposes a wrong token: the second drafter's
    branch (a copy-on-write view) wins, its pages are swapped into the sequence and
    decoding continues exactly as plain greedy decoding."""

    class Wrong:
        def propose(self, tokens, k):
            return [(int(tokens[-1]) + 1) % 100] * k

    model = _model()
    g = torch.Generator().manual_seed(4)
    base = torch.randint(0, model.cfg.vocab, (20,), generator=g).tolist()
    prompts = [base * 5]
    ref, _ = _run(model, "", prompts, 30)
    eng = LLMEngine(model, EngineConfig(num_blocks=256, max_model_len=1024))
    # the target as its own draft model behind a drafter that is always wrong: the
    # second branch (a copy-on-write view) is accepted and kept every step
    eng.spec = PoolSpecDecoder(eng, 6, DraftPool([Wrong(), ModelDrafter(model, 256)]))
    r = eng.add_request(prompts[0], SamplingParams(max_tokens=30))
    while eng.has_unfinished():
        eng.step()
    assert r.output == ref[0]
    st = eng.spec.stats()
    assert st["branch_wins"] > 0 and st["engines"][1]["wins"] > 0 and st["acceptance"] > 0.5
    eng.close()
