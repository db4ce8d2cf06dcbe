"""CPU end-to-end: BASELINE config 1 plumbing, engine restore equivalence, prefix cache
registration of restored blocks, worker save/restore API and the block manager."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "examples"))

from axropus_deploy_b200.amf import AmfManager, G1Pool  # noqa: E402
from axropus_deploy_b200.engine import BlockManager, EngineConfig, LLMEngine, SamplingParams, block_hashes  # noqa: E402
from axropus_deploy_b200.models.config import get_config  # noqa: E402
from axropus_deploy_b200.models.llama import LlamaModel  # noqa: E402


def test_config1_plumbing():
    import config1_cpu_plumbing as c1

    r = c1.run()
    assert r["raw_bit_exact"] and r["disk_reload_bit_exact"] and r["disk_lookup"] == "hit"
    assert r["fp8_max_abs_err"] < 0.25 and r["fp8_rel_err"] < 0.05
    assert r["int4_max_abs_err"] < 0.6 and r["int4_rel_err"] < 0.12
    assert r["fp8_bytes"] < 0.6 * r["raw_bytes"] and r["int4_bytes"] < 0.35 * r["raw_bytes"]


@pytest.fixture(scope="module")
def model():
    return LlamaModel(get_config("tiny"), "cpu", seed=0)


@pytest.mark.parametrize("fmt", ["raw", "fp8", "int4"])
def test_restore_then_decode_equals_cold(model, fmt):
    cfg = model.cfg
    pool = G1Pool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, fmt, slots_per_shard=64)
    amf = AmfManager(raw_pool=pool if fmt == "raw" else None, comp_pool=pool if fmt != "raw" else None)
    eng = LLMEngine(model, EngineConfig(num_blocks=160, max_model_len=1024), amf)
    g = torch.Generator().manual_seed(1)
    prefix = torch.randint(0, 32000, (512,), generator=g).tolist()
    p1 = prefix + torch.randint(0, 32000, (20,), generator=g).tolist()
    p2 = prefix + torch.randint(0, 32000, (33,), generator=g).tolist()
    cold = eng.add_request(p1, SamplingParams(max_tokens=6), amf_prefix_len=512)
    while eng.has_unfinished():
        eng.step()
    eng.evict_live_cache()
    warm = eng.add_request(p1, SamplingParams(max_tokens=6), amf_prefix_len=512)
    other = eng.add_request(p2, SamplingParams(max_tokens=6), amf_prefix_len=512)
    while eng.has_unfinished():
        eng.step()
    assert cold.amf_tier == "cold" and warm.amf_tier.startswith("g1") and warm.restored_tokens == 512
    assert other.amf_tier == "apc"  # restored blocks were registered and reused by the second request
    assert warm.output == cold.output
    st = eng.stats()
    assert st["amf"]["captures"] == 1 and st["restored_tokens"] == 512


def test_block_manager_prefix_cache():
    bm = BlockManager(8)
    toks = list(range(64))
    hs = block_hashes(toks)
    b = bm.allocate(4)
    bm.register_computed(b, hs)
    bm.release(b)
    assert bm.stats()["cached"] == 4
    got = bm.match_prefix(block_hashes(toks[:48] + [99] * 16))
    assert got == b[:3]
    bm.release(got)
    assert bm.evict_cached(0.5) == 2
    x = bm.allocate(8)
    assert len(set(x)) == 8 and bm.num_free() == 0
    with pytest.raises(MemoryError):
        bm.allocate(1)


def test_hashes_are_chained():
    a = block_hashes(list(range(48)))
    b = block_hashes([7] + list(range(1, 48)))
    assert all(x != y for x, y in zip(a, b))  # a change in block 0 changes every later hash


def test_amf_trace_lines(model, tmp_path, monkeypatch):
    """[AMF_KEY] / [AMF_MISS] / [AMF_SKIP] / [AMF_HIT] / [AMF_STATS] / [KORITH_RUN_SUMMARY]
    lines with the reference's field names, engine events as JSON lines."""
    import io
    import json

    events = tmp_path / "events.jsonl"
    monkeypatch.setenv("KORITH_ENGINE_EVENTS_PATH", str(events))
    cfg = model.cfg
    pool = G1Pool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, "raw", slots_per_shard=64)
    eng = LLMEngine(model, EngineConfig(num_blocks=160, max_model_len=1024, trace=True), AmfManager(raw_pool=pool))
    buf = io.StringIO()
    eng.trace.stream = buf
    prefix = list(range(7, 7 + 256))
    eng.generate([prefix + [1, 2, 3]], SamplingParams(max_tokens=3))
    eng.evict_live_cache()
    eng.generate([prefix + [4, 5, 6, 7]], SamplingParams(max_tokens=3))
    summ = eng.run_summary()
    out = buf.getvalue().splitlines()
    tags = [ln.split(" ", 1)[0] for ln in out]
    assert tags.count("[AMF_KEY]") == 2 and "[AMF_MISS]" in tags and "[AMF_HIT]" in tags and "[AMF_SKIP]" in tags
    assert tags[-2:] == ["[AMF_STATS]", "[KORITH_RUN_SUMMARY]"]
    hit = next(ln for ln in out if ln.startswith("[AMF_HIT]"))
    assert "prefix_tokens=256 skipped_tokens=256 baseline_ms=" in hit and " roi=" in hit
    assert out[0].startswith("[AMF_KEY] result=miss model_hash=") and " prompt_hash=" in out[0]
    assert summ["amf_hit"] == 1 and summ["tokens_generated"] == 6
    kinds = [json.loads(ln)["type"] for ln in events.read_text().splitlines()]
    assert kinds == ["amf_miss", "amf_hit"]


def test_admission_policy_prefers_hits_and_scales_budget(monkeypatch):
    from types import SimpleNamespace

    from axropus_deploy_b200.engine.scheduler import AdmissionPolicy

    monkeypatch.setenv("KORITH_VLLM_STARVATION_S", "100")
    pol = AdmissionPolicy()
    mk = lambda i, n, t: SimpleNamespace(prompt=[0] * n, t_arrival=t, params=SimpleNamespace(), i=i)
    w = [mk(0, 4000, 0.0), mk(1, 300, 0.1), mk(2, 5000, 0.2), mk(3, 800, 0.3)]
    held = {0: False, 1: False, 2: True, 3: False}
    order = [r.i for r in pol.order(w, lambda r: held[r.i], now=1.0)]
    assert order == [2, 1, 3, 0]  # the restorable prompt first, then shorter cold prompts
    old = mk(9, 9000, -200.0)  # starving: goes first whatever its cost
    assert pol.order(w + [old], lambda r: held.get(r.i, False), now=1.0)[0].i == 9
    assert pol.budget(16384, decoding=10, max_batch=64, head_is_hit=False) == 16384
    assert pol.budget(16384, decoding=60, max_batch=64, head_is_hit=False) == 12288
    assert pol.budget(16384, decoding=60, max_batch=64, head_is_hit=True) == 16384
    monkeypatch.setenv("KORITH_VLLM_DECODE_FIRST", "0")
    off = AdmissionPolicy()
    assert [r.i for r in off.order(w, lambda r: True)] == [0, 1, 2, 3]


def test_scheduler_trace_lines(model, tmp_path, monkeypatch):
    """KORITH_VLLM_SCHED_TRACE_PATH / _EVERY: every N-th admission round of a running engine
    appends one JSON line describing the queue."""
    import json

    path = tmp_path / "sched.jsonl"
    monkeypatch.setenv("KORITH_VLLM_SCHED_TRACE_PATH", str(path))
    monkeypatch.setenv("KORITH_VLLM_SCHED_TRACE_EVERY", "2")
    eng = LLMEngine(model, EngineConfig(num_blocks=64, max_model_len=512, max_batch=4))
    g = torch.Generator().manual_seed(7)
    eng.generate([torch.randint(0, 32000, (40,), generator=g).tolist() for _ in range(3)], SamplingParams(max_tokens=5))
    lines = [json.loads(x) for x in path.read_text().splitlines()]
    assert lines and all(x["round"] % 2 == 0 for x in lines)
    assert {"waiting", "decoding", "budget_tokens", "head_is_hit", "admitted", "held_waiting"} <= set(lines[0])
    assert sum(x["admitted"] for x in lines) <= 3 and eng.policy.rounds >= 2 * len(lines)


def test_prefill_graph_runner_padding_matches_eager(model):
    """The graph runner's padded one-sequence prefill (bucketed token count, slot -1
    padding, device-side lengths) gives the same tokens as the plain prefill. On CPU the
    padded step runs eagerly; on a GPU the same step is what the CUDA graph replays."""
    from axropus_deploy_b200.engine.cuda_graph import PrefillGraphRunner

    g = torch.Generator().manual_seed(3)
    prefix = torch.randint(0, 32000, (256,), generator=g).tolist()
    prompts = [prefix + torch.randint(0, 32000, (n,), generator=g).tolist() for n in (37, 100)]
    ref = LLMEngine(model, EngineConfig(num_blocks=96, max_model_len=1024)).generate(prompts, SamplingParams(max_tokens=4))
    eng = LLMEngine(model, EngineConfig(num_blocks=96, max_model_len=1024))
    eng._prefill_graphs = PrefillGraphRunner(eng, max_tokens=512)
    out = [eng.generate([p], SamplingParams(max_tokens=4))[0] for p in prompts]  # one sequence per prefill
    assert out == ref
    assert eng._prefill_graphs.stat["eager"] >= 1
    # the second prompt reuses the first one's cached prefix: its prefill is the 100-token suffix
    assert eng.stat["local_cached_tokens"] == 256


def test_mixed_steps_match_separate_forwards(model):
    """Prompts admitted while others decode run in one forward with the decode rows
    (mixed step); the generated tokens equal those of separate prefill and decode forwards."""
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, model.cfg.vocab, (n,), generator=g).tolist() for n in (40, 70, 33, 90, 51)]
    sp = SamplingParams(max_tokens=6)

    def run(mixed: bool):
        # a small prefill budget admits one prompt per step, so later prompts join running decodes
        eng = LLMEngine(model, EngineConfig(num_blocks=128, max_model_len=512, max_prefill_tokens=64,
                                            mixed_batch=mixed))
        reqs = [eng.add_request(p, sp) for p in prompts]
        while eng.has_unfinished():
            eng.step()
        return [r.output for r in reqs], eng.stat["mixed_steps"]

    ref, n_ref = run(False)
    out, n_mixed = run(True)
    assert n_ref == 0 and n_mixed > 0
    assert out == ref


def test_chunked_prefill_matches_whole_prompts(model):
    """While others decode, long prompts are prefilled in chunks over several mixed steps;
    the generated tokens equal those of whole-prompt prefills, and a prompt restored
    from the AMF pool after a chunked cold run gives the cold run's tokens."""
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, model.cfg.vocab, (n,), generator=g).tolist() for n in (30, 200, 170, 260)]
    sp = SamplingParams(max_tokens=5)

    def run(chunk: int, amf=None):
        eng = LLMEngine(model, EngineConfig(num_blocks=160, max_model_len=512, max_prefill_tokens=64,
                                            prefill_chunk=chunk), amf)
        reqs = [eng.add_request(p, sp, amf_prefix_len=len(p) // 16 * 16) for p in prompts]
        while eng.has_unfinished():
            eng.step()
        return [r.output for r in reqs], eng

    ref, e0 = run(0)
    pool = G1Pool(model.num_layers, model.cfg.num_kv_heads, model.cfg.head_dim, "raw", slots_per_shard=128,
                  device="cpu")
    out, e1 = run(48, AmfManager(raw_pool=pool, min_tokens=32))
    assert e0.stat["chunked_prefills"] == 0 and e1.stat["chunked_prefills"] > 0
    assert out == ref
    # the chunked cold prefills were captured whole: a fresh engine restores them
    eng = LLMEngine(model, EngineConfig(num_blocks=160, max_model_len=512), AmfManager(raw_pool=pool, min_tokens=32))
    r = eng.add_request(prompts[3], sp, amf_prefix_len=len(prompts[3]) // 16 * 16)
    while eng.has_unfinished():
        eng.step()
    assert r.amf_tier.startswith("g1") and r.output == ref[3]
