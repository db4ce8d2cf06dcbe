"""One cold prefill of Llama-3-8B (``--tokens`` new tokens, default 8320 = the headline
bench's 8 K prefix + 128-token suffix), device-timed: the whole forward and its parts.

    python benchmarks/prefill_step.py [--tokens 8320] [--reps 5]
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
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    cfg = get_config(args.model)
    T = args.tokens
    model = LlamaModel(cfg, dev, seed=0)
    pages = (T + 15) // 16
    cache = KVCache(cfg.num_layers, pages + 4, cfg.num_kv_heads, cfg.head_dim, "bf16", dev)
    bt = torch.arange(pages, dtype=torch.int32, device=dev)[None]
    pos = torch.arange(T, dtype=torch.int32, device=dev)
    toks = torch.randint(0, cfg.vocab, (T,), dtype=torch.int32, device=dev)
    meta = AttnMeta(mode="prefill", positions=pos, slots=pos.clone(), block_table=bt,
                    seq_lens=torch.tensor([T], dtype=torch.int32, device=dev),
                    cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), max_q=T, max_seq_len=T,
                    logits_idx=torch.tensor([T - 1], dtype=torch.int32, device=dev))
    for _ in range(2):
        model.forward(toks, meta, cache)
    torch.cuda.synchronize()
    if args.prof:
        torch.cuda.nvtx.range_push("prefill_step")
        model.forward(toks, meta, cache)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        print(json.dumps({"tokens": T, "prof": True}))
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
    q = torch.randn(T, cfg.num_heads, cfg.head_dim, device=dev).to(torch.bfloat16)
    at = []
    for _ in range(args.reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.prefill_attention(q, cache, 0, bt, meta.cu_q, meta.seq_lens, T, max_seq_len=T)
        e1.record()
        e1.synchronize()
        at.append(e0.elapsed_time(e1))
    attn_flop = 2.0 * T * T * cfg.head_dim * cfg.num_heads  # causal: half of 4 T^2 d per head
    gemm_flop = 2.0 * T * (cfg.param_count() - 2 * cfg.vocab * cfg.hidden) / 1.0
    out = {"tokens": T, "forward_ms": round(statistics.median(ts), 2),
           "attn_layer_ms": round(statistics.median(at), 3),
           "attn_tflops": round(attn_flop / (statistics.median(at) * 1e-3) / 1e12, 1),
           "gemm_tflop_per_forward": round(gemm_flop / 1e12, 1)}
    from axropus_deploy_b200.ops.gemm import check_errors

    assert check_errors(dev) == 0
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
