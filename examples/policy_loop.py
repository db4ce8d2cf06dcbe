"""The policy layer steering a live engine: curriculum workloads go through LLMEngine with
AMF (G1 pool); before each request the adaptive policy decides cache admission from the
engine's state vector, the executor applies it (switching AMF capture), and the outcome
(hit on an admitted prefix or not) is fed back and logged in the reward ledger.

Runs on cuda:0 when present, else on the CPU with a tiny model. Prints one JSON line.

    python examples/policy_loop.py [--levels 0 3] [--requests 24]
"""
import argparse
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from axropus_deploy_b200.amf import AmfManager, G1Pool  # noqa: E402
from axropus_deploy_b200.engine import EngineConfig, LLMEngine, SamplingParams  # noqa: E402
from axropus_deploy_b200.models.config import get_config  # noqa: E402
from axropus_deploy_b200.models.llama import LlamaModel  # noqa: E402
from axropus_deploy_b200.policy import (AdaptivePolicy, DecisionExecutor, RewardLedger, StateCollector,  # noqa: E402
                                        curriculum)


def run(levels=(0, 3), n_requests: int = 24, prefix_len: int = 128) -> dict:
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    cfg = get_config("tiny128" if dev == "cuda" else "tiny")
    model = LlamaModel(cfg, dev, seed=0)
    pool = G1Pool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, "raw", slots_per_shard=64,
                  **({"device": torch.device(dev)} if dev == "cuda" else {}))
    amf = AmfManager(raw_pool=pool, min_tokens=64)
    eng = LLMEngine(model, EngineConfig(num_blocks=256, max_model_len=1024, max_batch=8), amf)
    collector, policy, ledger = StateCollector(eng), AdaptivePolicy(), RewardLedger()
    executor = DecisionExecutor(amf=amf)
    out = {"device": dev, "levels": {}}
    for lv in levels:
        wl = curriculum(lv, n_requests, vocab=cfg.vocab, seed=lv)
        hits = 0
        for q in wl.requests:
            prompt = q["prompt"][:prefix_len] + q["prompt"][-16:]  # keep the example small
            v = collector.sample()
            d = policy.decide(v, q["tenant"], str(hash(tuple(prompt[:prefix_len]))))
            executor.execute(d, v)
            did = ledger.record_decision(d, v, q["tenant"])
            eng.evict_live_cache()  # only the AMF tiers can serve a repeat
            r = eng.add_request(prompt, SamplingParams(max_tokens=2), amf_prefix_len=prefix_len)
            while eng.has_unfinished():
                eng.step()
            hit = r.amf_tier != "cold"
            hits += hit
            if hit and d.cache_admission:
                ledger.record_outcome(did, "hit_admitted")
            elif d.cache_admission:
                ledger.record_outcome(did, "miss_never_reused")
            collector.record_lookup(hit, savings_ms=1.0 if hit else 0.0)
            policy.record_outcome(str(hash(tuple(prompt[:prefix_len]))), q["tenant"], d.spec_decode_depth,
                                  d.cache_admission, hit, 0.0)
        out["levels"][lv] = {"requests": len(wl.requests), "amf_hits": hits, "reuse": round(wl.reuse, 2),
                             "admit_now": executor.applied.cache_admission if executor.applied else None}
    out["rewards"] = ledger.summary()
    out["policy"] = policy.stat
    eng.close()
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--levels", type=int, nargs="+", default=[0, 3])
    ap.add_argument("--requests", type=int, default=24)
    a = ap.parse_args()
    print(json.dumps(run(tuple(a.levels), a.requests), default=str))
