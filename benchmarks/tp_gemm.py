"""Fused tensor-parallel GEMMs (all-gather -> GEMM, GEMM -> reduce-scatter) against the
NCCL + cuBLAS composition of the same layer, on the Llama-3-70B TP projections.

Run one process per GPU:

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        benchmarks/tp_gemm.py [--check-only] [--tokens 8192] [--iters 20]

Every rank checks the fused outputs against a float32 reference of the same layer (all
ranks generate every rank's inputs from fixed seeds, so no gather is needed), then times
both implementations with CUDA events (max over ranks) and rank 0 prints one JSON line
per layer. Inputs of each timed iteration rotate through buffers larger than L2.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from axropus_deploy_b200.ops.gemm import check_errors  # noqa: E402
from axropus_deploy_b200.parallel.dist import all_reduce_max, barrier, init_distributed, shutdown  # noqa: E402
from axropus_deploy_b200.parallel.tp import TpGemm, ag_gemm_nccl, gemm_rs_nccl  # noqa: E402

HIDDEN, INTER, KV = 8192, 28672, 1024  # Llama-3-70B


def _gen(shape, seed, device, scale=1.0):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=device) * scale).to(torch.bfloat16)


def _rel_err(x: torch.Tensor, ref: torch.Tensor) -> float:
    return float((x.float() - ref).norm() / ref.norm().clamp_min(1e-6))


def _time(fn, iters, info):
    for _ in range(3):
        fn(0)
    barrier(info)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(iters):
        fn(i)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / iters
    barrier(info)
    return all_reduce_max(ms, info)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192, help="tokens of the whole TP group (rows of the layer)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--check-only", action="store_true")
    ap.add_argument("--small", action="store_true", help="small shapes for a quick numerics check")
    args = ap.parse_args()
    info = init_distributed(timeout_s=60)
    W, R, dev = info.world, info.rank, info.device
    hidden, inter, kv = (1024, 2048, 256) if args.small else (HIDDEN, INTER, KV)
    tokens = args.tokens if not args.small else 256 * W
    rows = tokens // W
    n_qkv = (hidden + 2 * kv) // W
    n_up = 2 * inter // W
    k_o, k_down = hidden // W, inter // W
    tp = TpGemm(info, rows, hidden, hidden)
    results = []
    ok_all = True

    # ---- all-gather -> GEMM (qkv projection, gate/up projection)
    for name, n in (("ag_qkv", n_qkv), ("ag_gate_up", n_up)):
        x_full = _gen((tokens, hidden), 1, dev)
        w = _gen((n, hidden), 100 + R, dev, hidden ** -0.5)
        y = tp.ag_gemm(x_full[R * rows:(R + 1) * rows].contiguous(), w)
        torch.cuda.synchronize()
        ref = x_full.float() @ w.float().t()
        err = _rel_err(y, ref)
        ok = err < 2e-2 and check_errors(dev) == 0
        ok_all &= ok
        rec = {"layer": name, "world": W, "tokens": tokens, "n": n, "k": hidden, "rel_err": err, "ok": ok}
        if not args.check_only:
            nbuf = max(2, (256 << 20) // (rows * hidden * 2) + 1)
            xs = [_gen((rows, hidden), 7 + i, dev) for i in range(nbuf)]
            outs = [torch.empty(tokens, n, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            fused = _time(lambda i: tp.ag_gemm(xs[i % nbuf], w, outs[i & 1]), args.iters, info)
            base = _time(lambda i: ag_gemm_nccl(xs[i % nbuf], w, W), args.iters, info)
            flops = 2.0 * tokens * n * hidden
            rec.update(fused_ms=fused, nccl_cublas_ms=base, fused_tflops=flops / fused / 1e9,
                       speedup=base / fused)
        results.append(rec)

    # ---- GEMM -> reduce-scatter (o projection, down projection)
    for name, k in (("rs_o", k_o), ("rs_down", k_down)):
        a = _gen((tokens, k), 200 + R, dev)
        w = _gen((hidden, k), 300 + R, dev, k ** -0.5)
        y = tp.gemm_rs(a, w)
        torch.cuda.synchronize()
        ref = torch.zeros(rows, hidden, device=dev)
        for p in range(W):
            ap_ = _gen((tokens, k), 200 + p, dev)[R * rows:(R + 1) * rows]
            wp = _gen((hidden, k), 300 + p, dev, k ** -0.5)
            # each partial is rounded to bf16 before the sum, as in the fused kernel
            ref += (ap_.float() @ wp.float().t()).to(torch.bfloat16).float()
        err = _rel_err(y, ref)
        ok = err < 2e-2 and check_errors(dev) == 0
        ok_all &= ok
        rec = {"layer": name, "world": W, "tokens": tokens, "n": hidden, "k": k, "rel_err": err, "ok": ok}
        if not args.check_only:
            nbuf = max(2, (256 << 20) // (tokens * k * 2) + 1)
            As = [_gen((tokens, k), 17 + i, dev) for i in range(nbuf)]
            outs = [torch.empty(rows, hidden, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            fused = _time(lambda i: tp.gemm_rs(As[i % nbuf], w, outs[i & 1]), args.iters, info)
            base = _time(lambda i: gemm_rs_nccl(As[i % nbuf], w, W), args.iters, info)
            flops = 2.0 * tokens * hidden * k
            rec.update(fused_ms=fused, nccl_cublas_ms=base, fused_tflops=flops / fused / 1e9,
                       speedup=base / fused)
        results.append(rec)

    torch.cuda.synchronize()
    if R == 0:
        for rec in results:
            print(json.dumps(rec), flush=True)
        print("TP_CHECK", "ok" if ok_all else "FAILED", flush=True)
    del tp
    shutdown(info)
    if not ok_all:
        sys.exit(1)


if __name__ == "__main__":
    main()
