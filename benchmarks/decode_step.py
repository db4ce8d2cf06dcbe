"""One decode step of Llama-3-8B at the headline bench's shape, device-timed.

Builds the model (random-init weights) and a paged bf16 KV cache holding ``--batch``
sequences of ``--context`` tokens whose prefixes follow the bench's reuse pattern
(Zipf(1.1) over ``--prefixes`` prefixes, 10 % fresh), with random KV contents (the
attention values do not change the work). Times one decode forward, replayed from a CUDA
graph, with and without shared-prefix decode, L2 flushed before every replay; also the
attention of one layer alone.

    python benchmarks/decode_step.py [--batch 32] [--context 8448] [--reps 20]
"""
from __future__ import annotations

import argparse
import faulthandler
import json
import os
import statistics
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from axropus_deploy_b200 import ops  # noqa: E402
from axropus_deploy_b200.models.config import get_config  # noqa: E402
from axropus_deploy_b200.models.llama import AttnMeta, LlamaModel  # noqa: E402
from axropus_deploy_b200.ops.attention import CascadeMeta, cascade_groups, cascade_num_splits  # noqa: E402
from axropus_deploy_b200.ops.kvcache import KVCache  # noqa: E402


def build_tables(args, rng):
    """Block lists: reused prefixes share their blocks, fresh ones and suffixes own theirs."""
    pp = args.prefix_len // 16
    own_pages = (args.context - args.prefix_len + 15) // 16 + 1
    ranks = np.arange(1, args.prefixes + 1, dtype=np.float64)
    p = ranks ** -1.1
    p /= p.sum()
    next_block = 0
    prefix_blocks = {}
    lists = []
    for i in range(args.batch):
        if i % 10 == 9:  # fresh prefix
            key = ("fresh", i)
        else:
            key = int(rng.choice(args.prefixes, p=p))
        if key not in prefix_blocks:
            prefix_blocks[key] = list(range(next_block, next_block + pp))
            next_block += pp
        own = list(range(next_block, next_block + own_pages))
        next_block += own_pages
        lists.append(prefix_blocks[key] + own)
    return lists, next_block


def main():
    faulthandler.enable()  # a host crash prints where it happened
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--context", type=int, default=8448)
    ap.add_argument("--prefix-len", type=int, default=8192)
    ap.add_argument("--prefixes", type=int, default=64)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--prof", action="store_true",
                    help="run one eager decode forward inside the NVTX range 'decode_step' and stop "
                         "(for a per-kernel launch list under ncu --nvtx --nvtx-include decode_step/)")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    cfg = get_config(args.model)
    rng = np.random.default_rng(0)
    lists, nblocks = build_tables(args, rng)
    model = LlamaModel(cfg, dev, seed=0)
    cache = KVCache(cfg.num_layers, nblocks + 8, cfg.num_kv_heads, cfg.head_dim, "bf16", dev)
    cache.data.normal_(0, 1)
    B = args.batch
    width = max(len(x) for x in lists)
    bt = torch.zeros(B, width, dtype=torch.int32)
    for i, x in enumerate(lists):
        bt[i, :len(x)] = torch.tensor(x, dtype=torch.int32)
    bt = bt.to(dev)
    lens = torch.full((B,), args.context, dtype=torch.int32, device=dev)
    pos = lens - 1
    slots = torch.tensor([lists[i][(args.context - 1) // 16] * 16 + (args.context - 1) % 16 for i in range(B)],
                         dtype=torch.int32, device=dev)
    toks = torch.randint(0, cfg.vocab, (B,), dtype=torch.int32, device=dev)
    groups = cascade_groups(lists, 32, [args.prefix_len // 16] * B)
    q_index, cu, slen, first, row_of, ps = [], [0], [], [], [-1] * B, [0] * B
    for rows, shared in groups:
        for i in rows:
            row_of[i], ps[i] = len(q_index), shared
            q_index.append(i)
        cu.append(len(q_index))
        slen.append(shared * 16)
        first.append(rows[0])
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    casc = CascadeMeta(i32(q_index or [0]), i32(cu), i32(slen or [0]),
                       bt.index_select(0, torch.tensor(first or [0], device=dev)), i32(row_of), i32(ps),
                       max(len(r) for r, _ in groups) if groups else 1,
                       cascade_num_splits(len(groups), cfg.num_kv_heads, args.prefix_len, dev))
    S = ops.attention.decode_num_splits(B, cfg.num_kv_heads, (args.context + 15) // 16, dev, 0)
    flush = torch.empty(256 << 20, dtype=torch.int16, device=dev)
    out = {"batch": B, "context": args.context, "groups": [len(r) for r, _ in groups],
           "grouped_seqs": len(q_index), "decode_splits": S, "shared_splits": casc.num_splits}

    if args.prof:
        meta = AttnMeta(mode="decode", positions=pos, slots=slots, block_table=bt, seq_lens=lens,
                        max_seq_len=args.context, num_splits=S)
        for _ in range(2):
            model.forward(toks, meta, cache)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("decode_step")
        model.forward(toks, meta, cache)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        print(json.dumps(out), flush=True)
        return

    def timed(fn, reps):
        ts = []
        for _ in range(3):
            fn()
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    for name, c in (("plain", None), ("cascade", casc if groups else None)):  # cascade: opt-in engine path
        meta = AttnMeta(mode="decode", positions=pos, slots=slots, block_table=bt, seq_lens=lens,
                        max_seq_len=args.context, num_splits=S, cascade=c)
        q = torch.randn(B, cfg.num_heads, cfg.head_dim, device=dev).to(torch.bfloat16)
        out[f"attn_layer_ms_{name}"] = round(timed(lambda: ops.decode_attention(
            q, cache, 0, bt, lens, max_seq_len=args.context, num_splits=S, cascade=c), args.reps), 4)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                model.forward(toks, meta, cache)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            model.forward(toks, meta, cache)
        out[f"step_ms_{name}"] = round(timed(g.replay, args.reps), 3)
        del g
    kv_bytes = B * args.context * cfg.kv_bytes_per_token() / cfg.num_layers
    out["attn_plain_kv_tbs"] = round(kv_bytes / (out["attn_layer_ms_plain"] * 1e-3) / 1e12, 2)
    torch.cuda.synchronize()
    from axropus_deploy_b200.ops.gemm import check_errors

    assert check_errors(dev) == 0
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
