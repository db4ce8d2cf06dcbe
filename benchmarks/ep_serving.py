"""Expert-parallel agentic serving benchmark (Mixtral-8x7B, EP over the node's GPUs).

One process per GPU; attention is data-parallel (each GPU serves its own sessions) and the
MoE layers run expert-parallel through the fused dispatch / grouped GEMM / combine kernels,
all GPUs stepping in lockstep. AMF tiers: the FP8 G1 pool sharded across the GPUs by prefix
hash, with the CPU tier (LMCache-style) as fallback.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        benchmarks/ep_serving.py [--sessions 8 --turns 4]

Workload (per GPU): ``--sessions`` agentic sessions share a 4096-token system/tool prefix;
every turn extends a session's context by 300-1500 random tokens (after the previous turn's
output) and generates ``--out-tokens`` tokens; between turns half of the live KV cache is
evicted, so turns restore their context from the AMF tiers. TTFT of a request = device time
of the engine steps from the start of its turn to the step that produced its first token
(each step's time is the max over GPUs). Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from axropus_deploy_b200.amf.lmcache import LMCacheAdapter  # noqa: E402
from axropus_deploy_b200.amf.manager import AmfManager  # noqa: E402
from axropus_deploy_b200.amf.pool import PoolSlab  # noqa: E402
from axropus_deploy_b200.engine import EngineConfig, LLMEngine, SamplingParams  # noqa: E402
from axropus_deploy_b200.models.config import get_config  # noqa: E402
from axropus_deploy_b200.models.llama import LlamaModel  # noqa: E402
from axropus_deploy_b200.ops.kvcache import PAGE  # noqa: E402
from axropus_deploy_b200.parallel.dist import (all_gather_object, all_reduce_max, barrier,  # noqa: E402
                                               init_distributed, job_tag, shutdown)
from axropus_deploy_b200.parallel.sharded_pool import build_pool  # noqa: E402


def pct(xs, q):
    return float(np.percentile(np.asarray(xs), q)) if xs else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="mixtral-8x7b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--sessions", type=int, default=8, help="sessions per GPU")
    ap.add_argument("--turns", type=int, default=4)
    ap.add_argument("--prefix-len", type=int, default=4096)
    ap.add_argument("--ext-min", type=int, default=300)
    ap.add_argument("--ext-max", type=int, default=1500)
    ap.add_argument("--out-tokens", type=int, default=200)
    ap.add_argument("--evict", type=float, default=0.5)
    ap.add_argument("--pool-gb", type=float, default=20.0)
    ap.add_argument("--cpu-tier-gb", type=float, default=64.0)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()

    info = init_distributed(timeout_s=600.0)
    dev = info.device
    cfg = get_config(args.model)
    W = info.world
    max_ctx = args.prefix_len + args.turns * (args.ext_max + args.out_tokens) + PAGE
    # tokens of one prefill step (the MoE receive buffers are sized for all of them landing
    # on one GPU): a budget of 8192, or one whole context if that is longer
    max_prefill = max(8192, max_ctx)
    model = LlamaModel(cfg, dev, seed=args.seed, layers=args.layers, ep_info=info if W > 1 else None,
                       ep_max_tokens=max_prefill)
    L = model.num_layers
    nb = int(args.sessions * math.ceil(max_ctx / PAGE) * 1.15) + 64
    eng = LLMEngine(model, EngineConfig(num_blocks=nb, max_batch=args.sessions, max_prefill_tokens=max_prefill,
                                        max_model_len=max_ctx, lockstep=W > 1))
    chunk = PoolSlab.chunk_bytes(L, cfg.num_kv_heads, cfg.head_dim, "fp8")
    pool = build_pool(info, L, cfg.num_kv_heads, cfg.head_dim, "fp8", int(args.pool_gb * (1 << 30) // chunk),
                      job_tag() + "_ep")
    cpu = LMCacheAdapter(enabled=True, backend="cpu", max_bytes=int(args.cpu_tier_gb * (1 << 30)))
    eng.amf = AmfManager(comp_pool=pool, lmcache=cpu, lmcache_fallback=True, min_tokens=64)

    rng = np.random.default_rng(args.seed + 100 * info.rank)
    prefix = np.random.default_rng(args.seed).integers(0, cfg.vocab, args.prefix_len).tolist()
    ctx = [list(prefix) for _ in range(args.sessions)]

    def run_turn(timed: bool):
        """Submit one turn of every session; step all GPUs in lockstep until done."""
        reqs = []
        for s in range(args.sessions):
            ctx[s] += rng.integers(0, cfg.vocab, int(rng.integers(args.ext_min, args.ext_max + 1))).tolist()
            reqs.append(eng.add_request(list(ctx[s]), SamplingParams(max_tokens=args.out_tokens)))
        t_acc, ttft, step_ms = 0.0, {}, []
        while True:
            if all_reduce_max(1.0 if eng.has_unfinished() else 0.0, info) == 0.0:
                break
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            eng.step()
            e1.record()
            e1.synchronize()
            ms = all_reduce_max(e0.elapsed_time(e1), info)
            t_acc += ms
            step_ms.append(ms)
            for r in reqs:
                if r.output and r.req_id not in ttft:
                    ttft[r.req_id] = t_acc
        for s, r in enumerate(reqs):
            ctx[s] += r.output
        eng.evict_live_cache(args.evict)
        return reqs, ttft, t_acc

    # turn 0 populates (cold prefixes, captured); the rest are measured
    reqs, ttft, ms = run_turn(False)
    records, total_ms, out_tokens = [], 0.0, 0
    for t in range(1, args.turns):
        reqs, ttft, ms = run_turn(True)
        total_ms += ms
        for r in reqs:
            out_tokens += len(r.output)
            records.append({"turn": t, "tier": r.amf_tier, "ttft_ms": ttft.get(r.req_id),
                            "restored": r.restored_tokens, "cached": r.local_cached_tokens,
                            "prompt": len(r.prompt), "restore_ms": r.restore_ms})
    allrec = sum(all_gather_object(records, info), [])
    tok_all = sum(all_gather_object(out_tokens, info))
    amf = eng.amf.stats()
    barrier(info)
    if info.rank == 0:
        by_tier = {}
        for rec in allrec:
            by_tier.setdefault(rec["tier"], []).append(rec["ttft_ms"])
        restored = [r for r in allrec if r["restored"]]
        print(json.dumps({
            "metric": "EP agentic serving: TTFT by tier, output tok/s",
            "model": cfg.name, "layers": L, "ep": W, "sessions_per_gpu": args.sessions, "turns": args.turns,
            "prefix_len": args.prefix_len, "out_tokens": args.out_tokens, "evict": args.evict, "pool": "fp8",
            "cpu_tier": True,
            "ttft_ms": {tier: {"p50": pct(v, 50), "p99": pct(v, 99), "n": len(v)} for tier, v in by_tier.items()},
            "restored_tokens_p50": pct([r["restored"] for r in restored], 50),
            "restore_ms_p50": pct([r["restore_ms"] for r in restored], 50),
            "output_tok_s": tok_all / (total_ms * 1e-3) if total_ms else None,
            "amf_rank0": {k: amf[k] for k in ("hits_g1_pool", "hits_lmcache", "misses", "captures")},
            "timing": "per engine step: CUDA events, max over GPUs",
            "data": "synthetic random tokens, random-init weights",
        }), flush=True)
    eng.close()
    shutdown(info)


if __name__ == "__main__":
    main()
