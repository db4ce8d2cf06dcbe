"""One prefill forward of Llama-3-8B, device-timed: the whole forward and its attention.

Default: one cold prefill of ``--tokens`` new tokens (8320 = the headline bench's 8 K
prefix + 128-token suffix). With ``--batch B --context C``: the batched step the headline
bench runs for prefix-cache hits, B sequences of ``--tokens`` new tokens each over C
cached tokens (their KV is already in the cache; ``--distinct`` prefixes among them, the
rest share, as Zipf reuse does).

    python benchmarks/prefill_step.py [--tokens 8320] [--reps 5]
    python benchmarks/prefill_step.py --batch 30 --context 8192 --tokens 128 --distinct 8
    python benchmarks/prefill_step.py --prof   # one forward in NVTX range "prefill_step"
"""
from __future__ import annotations

import argparse
import faulthandler
import json
import os
import statistics
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from axropus_deploy_b200 import ops  # noqa: E402
from axropus_deploy_b200.models.config import get_config  # noqa: E402
from axropus_deploy_b200.models.llama import AttnMeta, LlamaModel  # noqa: E402
from axropus_deploy_b200.ops.kvcache import KVCache  # noqa: E402


def main():
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8320)
    ap.add_argument("--reps", type=int, default=5)
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--prof", action="store_true")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--context", type=int, default=0, help="cached tokens before each sequence's new ones (x16)")
    ap.add_argument("--distinct", type=int, default=0, help="distinct cached prefixes (0: one per sequence)")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    cfg = get_config(args.model)
    B, T, Cx = args.batch, args.tokens, args.context // 16 * 16
    model = LlamaModel(cfg, dev, seed=0)
    npre = args.distinct if args.distinct > 0 else B
    pp, sp = Cx // 16, (T + 15) // 16            # prefix pages, own pages per sequence
    pages = npre * pp + B * sp
    cache = KVCache(cfg.num_layers, pages + 4, cfg.num_kv_heads, cfg.head_dim, "bf16", dev)
    rows, slots, poss = [], [], []
    for b in range(B):
        pre = list(range((b % npre) * pp, (b % npre + 1) * pp))
        own = list(range(npre * pp + b * sp, npre * pp + (b + 1) * sp))
        rows.append(pre + own)
        p = torch.arange(Cx, Cx + T)
        blk = torch.tensor(rows[-1])[p // 16]
        slots.append(blk * 16 + p % 16)
        poss.append(p)
    width = max(len(r) for r in rows)
    bt = torch.tensor([r + [0] * (width - len(r)) for r in rows], dtype=torch.int32, device=dev)
    pos = torch.cat(poss).to(torch.int32).to(dev)
    slot_t = torch.cat(slots).to(torch.int32).to(dev)
    toks = torch.randint(0, cfg.vocab, (B * T,), dtype=torch.int32, device=dev)
    cu = torch.arange(0, B * T + 1, T, dtype=torch.int32, device=dev)
    L = Cx + T
    meta = AttnMeta(mode="prefill", positions=pos, slots=slot_t, block_table=bt,
                    seq_lens=torch.full((B,), L, dtype=torch.int32, device=dev),
                    cu_q=cu, max_q=T, max_seq_len=L, logits_idx=(cu[1:] - 1).contiguous())
    for _ in range(2):
        model.forward(toks, meta, cache)
    torch.cuda.synchronize()
    if args.prof:
        torch.cuda.nvtx.range_push("prefill_step")
        model.forward(toks, meta, cache)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        print(json.dumps({"tokens": T, "batch": B, "prof": True}))
        return
    ts = []
    for _ in range(args.reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        model.forward(toks, meta, cache)
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    # attention of one layer alone
    q = torch.randn(B * T, cfg.num_heads, cfg.head_dim, device=dev).to(torch.bfloat16)
    at = []
    for _ in range(args.reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.prefill_attention(q, cache, 0, bt, meta.cu_q, meta.seq_lens, T, max_seq_len=L)
        e1.record()
        e1.synchronize()
        at.append(e0.elapsed_time(e1))
    # causal over the new tokens, full over the cached ones: per head 4 d (T Cx + T^2 / 2)
    attn_flop = B * 4.0 * cfg.head_dim * cfg.num_heads * (T * Cx + T * T / 2)
    gemm_flop = 2.0 * B * T * (cfg.param_count() - 2 * cfg.vocab * cfg.hidden) / 1.0
    out = {"tokens": T, "batch": B, "context": Cx, "distinct": npre, "forward_ms": round(statistics.median(ts), 2),
           "attn_layer_ms": round(statistics.median(at), 3),
           "attn_tflops": round(attn_flop / (statistics.median(at) * 1e-3) / 1e12, 1),
           "gemm_tflop_per_forward": round(gemm_flop / 1e12, 1)}
    from axropus_deploy_b200.ops.gemm import check_errors

    assert check_errors(dev) == 0
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
