"""INT4 long-context decode (Llama-3-8B shape): sequences restored from 128K-token prefixes
held in the INT4 group-64 AMF pool, then decoded with split-KV flash-decode that reads the
INT4 pages directly.

    python benchmarks/long_context.py                      # one GPU
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        benchmarks/long_context.py                         # batch spread over 8 GPUs

The global batch (``--batch``, 32) is split over the GPUs; each sequence is restored
from its own prefix entry in the pool (sharded over the GPUs by prefix hash) through
the engine's AMF path (lookup -> restore into freshly allocated pages -> register as
computed -> prefill of the 16-token suffix -> ``--decode-tokens`` decode steps).

Prefilling 32 x 131072 tokens to create the pool entries would take far longer than the
measurement itself, so the entries hold synthetic INT4 pages (random codes and scales,
copied from a scratch cache) under the keys of random-token prefixes: restore and
decode move and read exactly the bytes a prefilled entry has. One GPU cannot hold 32
sequences of 128K INT4 KV plus their pool entries, so the batch per GPU is capped at
what fits (every sequence keeps its own entry) and the batch actually run is reported.

Also measured: restore latency of one 128K prefix from a raw bf16 pool entry into a
bf16 cache, for comparison.
"""
from __future__ import annotations

import argparse
import faulthandler
import json
import math
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from axropus_deploy_b200.amf.keys import pool_key, pool_key2  # noqa: E402
from axropus_deploy_b200.amf.manager import AmfManager  # noqa: E402
from axropus_deploy_b200.amf.pool import PoolSlab  # noqa: E402
from axropus_deploy_b200.engine import EngineConfig, LLMEngine, SamplingParams  # noqa: E402
from axropus_deploy_b200.models.config import get_config  # noqa: E402
from axropus_deploy_b200.models.llama import LlamaModel  # noqa: E402
from axropus_deploy_b200.ops.kvcache import PAGE, KVCache  # noqa: E402
from axropus_deploy_b200.parallel.dist import (all_gather_object, all_reduce_max, barrier,  # noqa: E402
                                               init_distributed, job_tag, shutdown)
from axropus_deploy_b200.parallel.sharded_pool import build_pool  # noqa: E402

GB = 1 << 30


def fill_random(cache: KVCache, seed: int) -> None:
    g = torch.Generator(device=cache.device).manual_seed(seed)
    if cache.fmt_name == "bf16":
        cache.data.normal_(generator=g)
    else:
        cache.data.random_(0, 256, generator=g)
        cache.meta[..., 0].uniform_(0.01, 0.03, generator=g)   # scale
        cache.meta[..., 1].uniform_(-0.1, 0.1, generator=g)    # zero point


def timed(fn, reps=3):
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    return min(ts)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--batch", type=int, default=32, help="global batch (split over the GPUs)")
    ap.add_argument("--prefix-len", type=int, default=131072)
    ap.add_argument("--suffix-len", type=int, default=16)
    ap.add_argument("--decode-tokens", type=int, default=512)
    ap.add_argument("--graphs", type=int, default=1)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--verbose", action="store_true", help="progress lines on stderr")
    args = ap.parse_args()
    faulthandler.enable()

    def note(msg):
        if args.verbose:
            print(f"[long_context] {msg}", file=sys.stderr, flush=True)

    info = init_distributed(timeout_s=900.0)
    dev, W, R = info.device, info.world, info.rank
    cfg = get_config(args.model)
    model = LlamaModel(cfg, dev, seed=args.seed)
    L, H, D = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
    pages = args.prefix_len // PAGE
    seq = args.prefix_len + args.suffix_len + args.decode_tokens
    blk_int4 = KVCache.bytes_per_block(L, H, D, "int4")
    b_local = args.batch // W + (1 if R < args.batch % W else 0)

    note("model ready")
    # ---- bf16 comparison first (its buffers are freed before the INT4 run)
    free0, _ = torch.cuda.mem_get_info(dev)
    bf_pages = pages
    bf_cache = KVCache(L, bf_pages + 16, H, D, "bf16", dev)
    bf_store = PoolSlab(bf_pages, L, H, D, "raw", dev)
    fill_random(bf_cache, 1)
    from axropus_deploy_b200.ops.kvcache import page_transfer

    blocks = torch.arange(bf_pages, dtype=torch.int32)
    page_transfer(bf_cache, blocks, bf_store, blocks)
    perm = torch.randperm(bf_pages, generator=torch.Generator().manual_seed(3)).to(torch.int32)
    bf_restore_ms = timed(lambda: page_transfer(bf_store, blocks, bf_cache, perm))
    del bf_cache, bf_store
    torch.cuda.empty_cache()

    note("bf16 restore measured")
    # ---- INT4 pool (sharded): every sequence gets its own prefix entry, on its own GPU's
    # shard (prefix keys drawn until their owner is that GPU). One GPU cannot hold 32
    # sequences of 128K INT4 KV plus their pool entries: the batch per GPU is capped at
    # what fits and reported.
    chunk = PoolSlab.chunk_bytes(L, H, D, "int4")
    per_seq = int(math.ceil(seq / PAGE) * 1.02) * blk_int4 + pages * chunk
    free, _ = torch.cuda.mem_get_info(dev)
    fit = max(1, int((free - 16 * GB) // per_seq))
    b_local = min(b_local, fit)
    counts = all_gather_object(b_local, info)
    batch = sum(counts)
    pool = build_pool(info, L, H, D, "int4", int(all_reduce_max(b_local, info)) * pages + 64, job_tag() + "_lc")
    rng = np.random.default_rng(args.seed + 5 + R)
    prefixes = []
    while len(prefixes) < b_local:
        p = rng.integers(0, cfg.vocab, args.prefix_len).tolist()
        if pool.owner(pool_key(p)) == R:
            prefixes.append(p)
    scratch = KVCache(L, 512, H, D, "int4", dev)
    fill_random(scratch, 2)
    src = (torch.arange(pages, dtype=torch.int32) % 512)
    for p in prefixes:
        assert pool.capture(pool_key(p), scratch, src, args.prefix_len, key2=pool_key2(p)), "pool full"
    del scratch
    torch.cuda.synchronize()
    barrier(info)

    note("pool populated")
    nb = int(b_local * math.ceil(seq / PAGE) * 1.02) + 64
    eng = LLMEngine(model, EngineConfig(num_blocks=nb, kv_fmt="int4", max_batch=max(1, b_local),
                                        max_prefill_tokens=4096, max_model_len=seq + PAGE,
                                        cuda_graphs=bool(args.graphs)))
    eng.amf = AmfManager(comp_pool=pool, min_tokens=64)
    reqs = []
    for p in prefixes:
        p = p + rng.integers(0, cfg.vocab, args.suffix_len).tolist()
        reqs.append(eng.add_request(p, SamplingParams(max_tokens=args.decode_tokens), amf_prefix_len=args.prefix_len))
    torch.cuda.synchronize()
    barrier(info)
    note("requests added")
    # admission (lookup + restore + register) and suffix prefill of every sequence
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    while any(r.state == "waiting" for r in reqs) or any(not r.output for r in reqs):
        eng.step()
    e1.record()
    e1.synchronize()
    admit_ms = all_reduce_max(e0.elapsed_time(e1), info)
    tiers = [r.amf_tier for r in reqs]
    restore_ms = [r.restore_ms for r in reqs]
    note("admitted")
    # decode: every remaining token of every sequence (the first decode step, which also
    # captures the decode CUDA graph of this batch size, is left out of the timing)
    eng.step()
    torch.cuda.synchronize()
    barrier(info)
    d0 = eng.stat["decode_tokens"]
    e0.record()
    while eng.has_unfinished():
        eng.step()
    e1.record()
    e1.synchronize()
    dec_ms = all_reduce_max(e0.elapsed_time(e1), info)
    dec_tok = sum(all_gather_object(eng.stat["decode_tokens"] - d0, info))
    all_tiers = sum(all_gather_object(tiers, info), [])
    all_restore = sum(all_gather_object(restore_ms, info), [])
    kv_int4_gb = b_local * seq * L * 2 * H * (D // 2 + D // 64 * 4) / 1e9
    eng.close()
    barrier(info)
    if R == 0:
        int4_prefix_bytes = pages * L * 2 * H * PAGE * (D // 2 + D // 64 * 4)
        print(json.dumps({
            "metric": "INT4 long-context decode tok/s; restore latency per 128K prefix (INT4 vs raw bf16)",
            "model": cfg.name, "gpus": W, "batch_requested": args.batch, "batch": batch, "batch_per_gpu": counts,
            "prefix_len": args.prefix_len, "decode_tokens": args.decode_tokens,
            "distinct_prefixes": batch, "hit_tiers": {t: all_tiers.count(t) for t in set(all_tiers)},
            "decode_tok_s": dec_tok / (dec_ms * 1e-3),
            "decode_ms_per_step": dec_ms / max(1, args.decode_tokens - 2),
            "live_int4_kv_gb_per_gpu": round(kv_int4_gb, 1),
            "restore_ms_per_128k_int4_p50": float(np.median(all_restore)),
            "restore_int4_gbps": int4_prefix_bytes / (float(np.median(all_restore)) * 1e-3) / 1e9,
            "admission_incl_restore_and_suffix_prefill_ms": admit_ms,
            "restore_ms_per_128k_bf16_raw": bf_restore_ms,
            "restore_bf16_gbps": pages * L * 2 * H * PAGE * D * 2 / (bf_restore_ms * 1e-3) / 1e9,
            "timing": "CUDA events, max over GPUs; restore_ms from the engine's admission path (host-synchronised)",
            "data": "pool entries hold synthetic INT4 pages under random-token prefix keys; random-init weights",
        }), flush=True)
    shutdown(info)


if __name__ == "__main__":
    main()
