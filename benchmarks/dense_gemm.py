"""Dense projections of Llama-3-8B: this framework's tcgen05 kernels (ops/dense.py) against
cuBLAS (torch.matmul) on the same shapes, CUDA-event timed, L2 flushed before every timed
launch (a 512 MB write), median of the repeats.

Reports per shape: time, weight-read bandwidth (bytes of W / time) and TFLOP/s, as a
fraction of the measured copy bandwidth and cuBLAS bf16 peak in MEASURED_PEAKS.json.

    python benchmarks/dense_gemm.py [--rows 1,32,128,256,1024,8320] [--reps 20]
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

from axropus_deploy_b200.ops import dense  # noqa: E402

SHAPES = {  # name: (N, K, epilogue)
    "qkv": (6144, 4096, "store"),
    "o": (4096, 4096, "resid"),
    "gate_up": (28672, 4096, "swiglu"),
    "down": (4096, 14336, "resid"),
    "lm_head": (128256, 4096, "store"),
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"]
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0


def timed(fn, flush, reps):
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


def main():
    faulthandler.enable()  # a host crash prints where it happened
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", default="1,32,128,256,1024,8320")
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--shapes", default=",".join(SHAPES))
    ap.add_argument("--chain", action="store_true",
                    help="time back-to-back launches over rotating weight copies (> 512 MB in all, so every "
                         "launch reads its weights from HBM), as in a decode step; per-launch average")
    ap.add_argument("--splits", default="0", help="comma list of forced split counts (0 = automatic)")
    args = ap.parse_args()
    if args.chain:
        return chain(args)
    dev = torch.device("cuda", 0)
    hbm, tflops = peaks()
    flush = torch.empty(256 << 20, dtype=torch.int16, device=dev)
    g = torch.Generator(device=dev).manual_seed(0)
    rows = [int(r) for r in args.rows.split(",")]
    out = []
    for name in args.shapes.split(","):
        N, K, epi = SHAPES[name]
        w = torch.empty(N, K, dtype=torch.bfloat16, device=dev).normal_(0, 0.02, generator=g)
        wt = w.t()  # cuBLAS on the same weights: x @ w^T
        dense.reserve(dev, [(N, K)])
        for M in rows:
            x = torch.empty(M, K, dtype=torch.bfloat16, device=dev).normal_(0, 1, generator=g)
            res = torch.empty(M, N, dtype=torch.bfloat16, device=dev).normal_(0, 1, generator=g)
            if epi == "resid":
                ours = lambda: dense.linear(x, w, "resid", out=res, res=res)  # noqa: E731
            else:
                ours = lambda: dense.linear(x, w, epi)  # noqa: E731
            ref = lambda: torch.matmul(x, wt)  # noqa: E731
            t_ours = timed(ours, flush, args.reps)
            t_ref = timed(ref, flush, args.reps)
            wbytes = N * K * 2
            flop = 2.0 * M * N * K
            from axropus_deploy_b200.ops._ext import cuda_ext
            row = {"shape": name, "M": M, "N": N, "K": K, "epilogue": epi,
                   "splits": cuda_ext().dense_stream_splits(M, N, K, dense.sm_count(dev)) if M <= 256 else 0,
                   "pair_clusters": cuda_ext().dense_pair_clusters(dev.index) if M > 256 else 0,
                   "ours_ms": round(t_ours, 4),
                   "cublas_ms": round(t_ref, 4), "speedup": round(t_ref / t_ours, 3),
                   "ours_weight_gbs": round(wbytes / t_ours / 1e6, 1),
                   "ours_tflops": round(flop / t_ours / 1e9, 1),
                   "frac_hbm": round(wbytes / t_ours / 1e6 / hbm, 3),
                   "frac_bf16": round(flop / t_ours / 1e9 / tflops, 3)}
            out.append(row)
            print(json.dumps(row), flush=True)
    torch.cuda.synchronize()
    from axropus_deploy_b200.ops.gemm import check_errors

    assert check_errors(dev) == 0


def chain(args):
    dev = torch.device("cuda", 0)
    hbm, _ = peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    for name in args.shapes.split(","):
        N, K, epi = SHAPES[name]
        copies = max(2, -(-(512 << 20) // (N * K * 2)))
        ws = [torch.empty(N, K, dtype=torch.bfloat16, device=dev).normal_(0, 0.02, generator=g) for _ in range(copies)]
        dense.reserve(dev, [(N, K)])
        for M in [int(r) for r in args.rows.split(",")]:
            x = torch.empty(M, K, dtype=torch.bfloat16, device=dev).normal_(0, 1, generator=g)
            res = torch.empty(M, N, dtype=torch.bfloat16, device=dev).normal_(0, 1, generator=g)
            variants = [("cublas", None)] + [(f"ours_s{s}", int(s)) for s in args.splits.split(",")]
            row = {"shape": name, "M": M, "N": N, "K": K, "copies": copies}
            for label, sp in variants:
                def run():
                    for w in ws:
                        if sp is None:
                            torch.matmul(x, w.t())
                        elif epi == "resid":
                            dense.linear(x, w, "resid", out=res, res=res, splits=sp)
                        else:
                            dense.linear(x, w, epi, splits=sp)
                for _ in range(2):
                    run()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(3):
                    run()
                e1.record()
                e1.synchronize()
                us = e0.elapsed_time(e1) * 1e3 / (3 * copies)
                row[label + "_us"] = round(us, 2)
                row[label + "_frac_hbm"] = round(N * K * 2 / (us * 1e-6) / 1e9 / hbm, 3)
            print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
