"""Prefill attention alone (ops.prefill_attention -> the tcgen05 kernel), CUDA-event timed
after warm-up, median of the repeats, as a fraction of the measured bf16 tensor peak
(MEASURED_PEAKS.json). FLOPs: per query row and head, 4 d (keys it sees); causal rows see
their prefix.

    python benchmarks/prefill_attn.py [--reps 10]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from axropus_deploy_b200 import ops  # noqa: E402
from axropus_deploy_b200.ops.kvcache import KVCache  # noqa: E402

# name: (sequences, new tokens each, cached tokens before them, q heads, kv heads, distinct prefixes)
CASES = {
    "8192x1 32/8": (1, 8192, 0, 32, 8, 1),
    "32768x1 8/1": (1, 32768, 0, 8, 1, 1),
    "4096x1 64/8": (1, 4096, 0, 64, 8, 1),
    "2048x4 32/8": (4, 2048, 0, 32, 8, 4),
    "128x30 over 8192 32/8": (30, 128, 8192, 32, 8, 8),
}


def peak() -> float:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"])
    except (OSError, KeyError, ValueError):
        return 1590.0


def run_case(name, B, T, C, Hq, Hkv, npre, reps, dev):
    pp, sp = C // 16, (T + 15) // 16
    pages = npre * pp + B * sp
    cache = KVCache(1, pages + 4, Hkv, 128, "bf16", dev)
    cache.data.normal_()
    rows = []
    for b in range(B):
        rows.append(list(range((b % npre) * pp, (b % npre + 1) * pp)) +
                    list(range(npre * pp + b * sp, npre * pp + (b + 1) * sp)))
    bt = torch.tensor(rows, dtype=torch.int32, device=dev)
    cu = torch.arange(0, B * T + 1, T, dtype=torch.int32, device=dev)
    sl = torch.full((B,), C + T, dtype=torch.int32, device=dev)
    q = torch.randn(B * T, Hq, 128, device=dev).to(torch.bfloat16)
    fn = lambda: ops.prefill_attention(q, cache, 0, bt, cu, sl, T, max_seq_len=C + T)  # noqa: E731
    for _ in range(3):
        fn()
    ts = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        ts.append(e0.elapsed_time(e1))
    ms = statistics.median(ts)
    flop = B * Hq * 4.0 * 128 * (T * C + T * (T + 1) / 2)
    tf = flop / (ms * 1e-3) / 1e12
    return {"case": name, "ms": round(ms, 4), "tflops": round(tf, 1), "frac_of_measured_bf16": round(tf / peak(), 3)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--cases", default=",".join(CASES))
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    for name in args.cases.split(","):
        print(json.dumps(run_case(name, *CASES[name], args.reps, dev)), flush=True)
    from axropus_deploy_b200.ops.gemm import check_errors

    assert check_errors(dev) == 0


if __name__ == "__main__":
    main()
