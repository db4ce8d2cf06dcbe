"""Engine on the GPU: an AMF hit restored from the G1 pool (raw bf16 and FP8) while the
suffix prefill is launched -- the restore is not synchronised on its own -- gives the cold
run's tokens (raw) and leaves no pin on the pool entry; the one-sequence prefill CUDA graph
gives the eager prefill's tokens."""
import pytest
import torch


def _engine(fmt, graphs):
    from axropus_deploy_b200.amf import AmfManager, G1Pool
    from axropus_deploy_b200.engine import EngineConfig, LLMEngine
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel

    dev = torch.device("cuda", 0)
    cfg = get_config("tiny128")
    model = LlamaModel(cfg, dev, seed=0)
    pool = G1Pool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, fmt, slots_per_shard=128, device=dev)
    amf = AmfManager(raw_pool=pool if fmt == "raw" else None, comp_pool=pool if fmt != "raw" else None, min_tokens=64)
    eng = LLMEngine(model, EngineConfig(num_blocks=512, max_model_len=2048, max_batch=8, cuda_graphs=graphs), amf)
    return eng, pool


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["raw", "fp8"])
@pytest.mark.parametrize("graphs", [False, True])
def test_restore_overlapped_with_prefill(fmt, graphs):
    from axropus_deploy_b200.engine import SamplingParams

    eng, pool = _engine(fmt, graphs)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, eng.model.cfg.vocab, (1000,), generator=g).tolist()
    cold = eng.add_request(prompt, SamplingParams(max_tokens=6), amf_prefix_len=960)
    while eng.has_unfinished():
        eng.step()
    for _ in range(2):  # the second warm run replays the captured prefill graph
        eng.evict_live_cache()
        warm = eng.add_request(prompt, SamplingParams(max_tokens=6), amf_prefix_len=960)
        while eng.has_unfinished():
            eng.step()
        torch.cuda.synchronize()
        assert warm.amf_tier.startswith("g1") and warm.restored_tokens == 960
        assert warm.restore_ms > 0
        if fmt == "raw":
            assert warm.output == cold.output
    pins = [sum(e["pins"]) if isinstance(e["pins"], (list, tuple)) else e["pins"]
            for s in range(pool.world) for e in pool.dir.entries(s)]
    assert pins and all(p == 0 for p in pins)
    if graphs:
        assert eng._prefill_graphs.stat["replays"] >= 2
    eng.close()


@pytest.mark.gpu
def test_pipelined_decode_matches_serial():
    """Decode pipelining (step t + 1 launched on device tokens before step t is read) gives
    the tokens of the serial loop: different lengths, a stop token, a request joining."""
    import torch

    from axropus_deploy_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel

    dev = torch.device("cuda", 0)
    model = LlamaModel(get_config("tiny128"), dev, seed=1)
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (40, 75, 130, 20)]

    def run(pipe, stop=()):
        eng = LLMEngine(model, EngineConfig(num_blocks=256, max_model_len=1024, max_batch=8, cuda_graphs=True,
                                            pipeline_decode=pipe))
        reqs = [eng.add_request(p, SamplingParams(max_tokens=m, stop_token_ids=stop))
                for p, m in zip(prompts[:3], (12, 5, 20))]
        for _ in range(3):
            eng.step()
        late = eng.add_request(prompts[3], SamplingParams(max_tokens=7, stop_token_ids=stop))
        while eng.has_unfinished():
            eng.step()
        out = [r.output for r in reqs + [late]]
        st = dict(eng.stat)
        eng.close()
        return out, st

    serial, st0 = run(False)
    piped, st = run(True)
    assert piped == serial and st["pipelined_decode_steps"] > 0
    # the late request joins the pipelined batch instead of decoding alone afterwards
    assert st["steps"] <= st0["steps"] + 1, (st["steps"], st0["steps"])
    stop = serial[2][4]  # a stop token in the middle of the longest request
    s2, _ = run(False, (stop,))
    p2, _ = run(True, (stop,))
    assert p2 == s2 and len(p2[2]) <= 5
