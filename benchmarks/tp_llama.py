"""Tensor-parallel serving benchmark (Llama-3-70B, TP over the node's GPUs, FP8 AMF pool).

One process per GPU:

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        benchmarks/tp_llama.py [--prefix-len 32768 --prefixes 32 --suffix-len 256 --out-tokens 256]

Workload: ``--prefixes`` distinct random-token prefixes; each is prefilled cold once
(TTFT cold, captured into this GPU's FP8 pool shard of its own KV heads), the live cache
is evicted, and requests reusing a prefix (uniform choice) plus a random suffix are
served (TTFT hit = restore from the pool + suffix prefill). Then ``--decode-batch``
requests decode ``--out-tokens`` tokens (decode tok/s). Times are device times (CUDA
events around each engine step), max over ranks. ``--tp-impl nccl`` runs the same
sequence-parallel layout with NCCL all-gather / reduce-scatter + cuBLAS instead of the
fused kernels, for comparison. Rank 0 prints one JSON line.
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

from axropus_deploy_b200.amf.manager import AmfManager  # noqa: E402
from axropus_deploy_b200.amf.pool import PoolSlab  # noqa: E402
from axropus_deploy_b200.engine import EngineConfig, LLMEngine, SamplingParams  # noqa: E402
from axropus_deploy_b200.models.config import get_config  # noqa: E402
from axropus_deploy_b200.models.llama_tp import TpLlamaModel  # noqa: E402
from axropus_deploy_b200.ops.kvcache import PAGE  # noqa: E402
from axropus_deploy_b200.parallel.dist import (DistInfo, all_reduce_max, barrier, init_distributed,  # noqa: E402
                                               job_tag, shutdown)
from axropus_deploy_b200.parallel.sharded_pool import build_pool  # noqa: E402


def pct(xs, q):
    return float(np.percentile(np.asarray(xs), q)) if xs else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-70b")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--prefix-len", type=int, default=32768)
    ap.add_argument("--prefixes", type=int, default=32)
    ap.add_argument("--suffix-len", type=int, default=256)
    ap.add_argument("--out-tokens", type=int, default=256)
    ap.add_argument("--hit-samples", type=int, default=8)
    ap.add_argument("--decode-batch", type=int, default=16)
    ap.add_argument("--pool", default="fp8", choices=["raw", "fp8", "int4"])
    ap.add_argument("--pool-gb", type=float, default=40.0)
    ap.add_argument("--tp-impl", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--graphs", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--nccl-samples", type=int, default=2,
                    help="cold prefills also timed with NCCL all-gather/reduce-scatter + cuBLAS")
    ap.add_argument("--check", action="store_true",
                    help="numerics only: TP model vs the dense model on every rank (tiny128)")
    args = ap.parse_args()
    if args.check:
        return check()

    info = init_distributed(timeout_s=600.0)
    dev = info.device
    cfg = get_config(args.model)
    max_tok = args.prefix_len + args.suffix_len + PAGE
    model = TpLlamaModel(cfg, info, seed=args.seed, layers=args.layers, max_tokens=max_tok,
                         fused=args.tp_impl == "fused")
    L = model.num_layers
    seq = args.prefix_len + args.suffix_len + args.out_tokens
    nb = int(max(args.decode_batch, 2) * math.ceil(seq / PAGE) * 1.1) + 64
    eng = LLMEngine(model, EngineConfig(num_blocks=nb, max_batch=max(args.decode_batch, 2),
                                        max_prefill_tokens=max_tok, max_model_len=seq + PAGE,
                                        cuda_graphs=bool(args.graphs)))
    # this GPU's pool shard holds its own KV heads of every captured prefix
    chunk = PoolSlab.chunk_bytes(L, model.hkv, cfg.head_dim, args.pool)
    slots = int(args.pool_gb * (1 << 30) // chunk)
    local = DistInfo(0, 1, 0, 1, dev)
    pool = build_pool(local, L, model.hkv, cfg.head_dim, args.pool, slots, f"{job_tag()}_tp{info.rank}")
    eng.amf = AmfManager(comp_pool=pool if args.pool != "raw" else None, raw_pool=pool if args.pool == "raw" else None,
                         min_tokens=64)

    rng = np.random.default_rng(args.seed + 17)
    prefixes = [rng.integers(0, cfg.vocab, args.prefix_len).tolist() for _ in range(args.prefixes)]

    def suffix():
        return rng.integers(0, cfg.vocab, args.suffix_len).tolist()

    def timed_first_token(prompt, max_tokens=1):
        """Device time of the step that admits + prefills the request (its TTFT)."""
        torch.cuda.synchronize()
        barrier(info)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r = eng.add_request(prompt, SamplingParams(max_tokens=max_tokens), amf_prefix_len=args.prefix_len)
        e0.record()
        eng.step()
        e1.record()
        e1.synchronize()
        while eng.has_unfinished():
            eng.step()
        return r, all_reduce_max(e0.elapsed_time(e1), info)

    # warm-up: one short cold request + its hit (compiles graphs, allocator, NCCL)
    w = rng.integers(0, cfg.vocab, 2048).tolist()
    timed_first_token(w + suffix())
    eng.evict_live_cache()
    timed_first_token(w + suffix())

    ttft_cold, ttft_hit, restore_ms, tiers = [], [], [], {}
    for pf in prefixes:  # every prefix once cold: TTFT cold + capture into the pool
        r, ms = timed_first_token(pf + suffix())
        ttft_cold.append(ms)
        eng.evict_live_cache()
    for i in range(args.hit_samples):
        eng.evict_live_cache()
        r, ms = timed_first_token(prefixes[int(rng.integers(0, len(prefixes)))] + suffix())
        tiers[r.amf_tier] = tiers.get(r.amf_tier, 0) + 1
        if r.amf_tier.startswith("g1"):
            ttft_hit.append(ms)
            restore_ms.append(all_reduce_max(r.restore_ms, info))

    # restore bandwidth, device-timed: one prefix from this GPU's pool shard into the cache
    hit = eng.amf.lookup(np.asarray(prefixes[0] + [0] * 16, dtype=np.int64).astype(np.uint32).view(np.int32),
                         args.prefix_len)
    rest_gbps = None
    if hit is not None:
        blocks = torch.tensor(eng.bm.allocate(hit.n_pages), dtype=torch.int32)
        times = []
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            hit.restore(eng.cache, blocks)
            e1.record()
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        hit.release()
        eng.bm.release(blocks.tolist())
        # bytes of KV materialised in this GPU's live cache (bf16, its own heads)
        kv = hit.n_tokens * L * 2 * model.hkv * cfg.head_dim * 2
        rest_gbps = kv / (min(times[1:]) * 1e-3) / 1e9
    have = 1 if hit is not None else 0
    from axropus_deploy_b200.parallel.dist import all_reduce_min

    if all_reduce_min(have, info) == 0:
        rest_gbps = None

    # the same cold prefill with the collectives done by NCCL (+ cuBLAS GEMMs)
    ttft_cold_nccl = []
    if args.tp_impl == "fused" and args.nccl_samples > 0:
        model.fused = False
        for i in range(args.nccl_samples):
            eng.evict_live_cache()
            eng.amf.disable_restore = True
            r, ms = timed_first_token(prefixes[i % len(prefixes)] + suffix())
            eng.amf.disable_restore = False
            ttft_cold_nccl.append(ms)
        model.fused = True

    # decode throughput: a batch of hit requests, all tokens generated (one untimed
    # batch first so the decode graphs of this batch size are captured)
    for timed in (False, True):
        eng.evict_live_cache()
        n_out = args.out_tokens if timed else 4
        reqs = [eng.add_request(prefixes[i % len(prefixes)] + suffix(), SamplingParams(max_tokens=n_out),
                                amf_prefix_len=args.prefix_len) for i in range(args.decode_batch)]
        if not timed:
            while eng.has_unfinished():
                eng.step()
    eng.evict_live_cache()
    reqs = [eng.add_request(prefixes[i % len(prefixes)] + suffix(), SamplingParams(max_tokens=args.out_tokens),
                            amf_prefix_len=args.prefix_len) for i in range(args.decode_batch)]
    eng.step()  # admission + prefill of the whole batch
    torch.cuda.synchronize()
    barrier(info)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0 = eng.stat["decode_tokens"]
    e0.record()
    while eng.has_unfinished():
        eng.step()
    e1.record()
    e1.synchronize()
    dec_ms = all_reduce_max(e0.elapsed_time(e1), info)
    dec_tokens = eng.stat["decode_tokens"] - d0
    assert all(len(r.output) == args.out_tokens for r in reqs)
    eng.close()
    torch.cuda.synchronize()
    barrier(info)
    if info.rank == 0:
        print(json.dumps({
            "metric": "TP serving: TTFT hit vs cold, restore GB/s, decode tok/s",
            "model": cfg.name, "layers": L, "tp": info.world, "tp_impl": args.tp_impl,
            "prefix_len": args.prefix_len, "prefixes": args.prefixes, "suffix_len": args.suffix_len,
            "pool": args.pool, "pool_gb_per_gpu": args.pool_gb,
            "ttft_cold_ms": {"p50": pct(ttft_cold, 50), "p99": pct(ttft_cold, 99), "n": len(ttft_cold)},
            "ttft_cold_nccl_ms": {"p50": pct(ttft_cold_nccl, 50), "n": len(ttft_cold_nccl)},
            "ttft_hit_ms": {"p50": pct(ttft_hit, 50), "p99": pct(ttft_hit, 99), "n": len(ttft_hit)},
            "restore_ms_p50": pct(restore_ms, 50), "restore_gbps_per_gpu": rest_gbps, "hit_tiers": tiers,
            "decode_batch": args.decode_batch, "decode_tokens": dec_tokens,
            "decode_tok_s": dec_tokens / (dec_ms * 1e-3),
            "timing": "CUDA events per engine step, max over ranks",
            "data": "synthetic random tokens, random-init weights",
        }), flush=True)
    shutdown(info)


def check():
    """TP model (fused AG/RS prefill + replicated decode) vs the dense model, logits."""
    from axropus_deploy_b200.models.llama import AttnMeta, LlamaModel
    from axropus_deploy_b200.ops.kvcache import KVCache

    info = init_distributed(timeout_s=120.0)
    dev = info.device
    cfg = get_config("tiny128")
    dense = LlamaModel(cfg, dev, seed=3, init_std=0.05)
    tp = TpLlamaModel(cfg, info, dense=dense, max_tokens=2048, sp_min_tokens=256)
    T = 700
    tokens = torch.randint(0, cfg.vocab, (T,), generator=torch.Generator().manual_seed(1)).to(dev, torch.int32)
    errs = {}
    for name, m, heads in (("dense", dense, cfg.num_kv_heads), ("tp", tp, tp.hkv)):
        cache = KVCache(m.num_layers, 64, heads, cfg.head_dim, "bf16", dev)
        bt = torch.arange(64, dtype=torch.int32, device=dev)[None]
        pos = torch.arange(T, dtype=torch.int32, device=dev)
        meta = AttnMeta("prefill", pos, pos, bt, torch.tensor([T], dtype=torch.int32, device=dev),
                        cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), max_q=T, max_seq_len=T,
                        logits_idx=torch.tensor([T - 1], dtype=torch.int32, device=dev))
        lp = m.forward(tokens, meta, cache)
        p1 = torch.tensor([T], dtype=torch.int32, device=dev)
        dmeta = AttnMeta("decode", p1, p1, bt, torch.tensor([T + 1], dtype=torch.int32, device=dev), max_seq_len=T + 1)
        ld = m.forward(tokens[:1], dmeta, cache)
        errs[name] = (lp, ld)
    rel = [float((errs["tp"][i] - errs["dense"][i]).norm() / errs["dense"][i].norm()) for i in range(2)]
    ok = max(rel) < 3e-2
    if info.rank == 0:
        print(json.dumps({"check": "tp_vs_dense", "world": info.world, "rel_prefill": rel[0], "rel_decode": rel[1],
                          "ok": ok}), flush=True)
        print("TP_LLAMA_CHECK", "ok" if ok else "FAILED", flush=True)
    shutdown(info)
    if not ok:
        sys.exit(1)


if __name__ == "__main__":
    main()
