"""Expert-parallel MoE layer (Mixtral-8x7B shapes): fused dispatch / grouped tcgen05 expert
GEMMs / combine against the NCCL all-to-all + per-expert cuBLAS composition of the same layer.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        benchmarks/ep_moe.py [--check] [--tokens 4096] [--iters 10]

Every rank routes its own tokens (top-2 of 8). ``--check`` compares the fused layer with a
float32 reference on every rank (each rank regenerates every expert's weights from its seed)
and prints ``EP_CHECK ok``. Timing: CUDA events, max over ranks; rank 0 prints JSON lines.
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
from axropus_deploy_b200.parallel.ep import EpMoE, experts_reference, route  # noqa: E402


def expert_weights(e, H, F, dev, std=0.02):
    g = torch.Generator(device=dev).manual_seed(1000 + e)
    w13 = (torch.randn(2 * F, H, generator=g, device=dev) * std).to(torch.bfloat16)
    w2 = (torch.randn(H, F, generator=g, device=dev) * std).to(torch.bfloat16)
    return w13, w2


def nccl_layer(x, idx, w, w13_local, w2_local, E_l, W, rank):
    """all_to_all_single dispatch + per-expert cuBLAS + all_to_all_single combine."""
    T, K = idx.shape
    flat = idx.view(-1).long()
    dst = flat // E_l
    order = torch.argsort(dst, stable=True)
    send_counts = torch.bincount(dst, minlength=W)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    xs = x[order // K]
    xr = torch.empty(sum(rc), x.shape[1], dtype=x.dtype, device=x.device)
    dist.all_to_all_single(xr, xs, rc, sc)
    er = torch.empty(sum(rc), dtype=torch.int64, device=x.device)
    dist.all_to_all_single(er, flat[order].contiguous(), rc, sc)
    yr = torch.empty_like(xr)
    le = er - rank * E_l
    F = w2_local.shape[2]
    for e in range(E_l):
        sel = (le == e).nonzero(as_tuple=True)[0]
        if sel.numel():
            gu = xr[sel] @ w13_local[e].t()
            g, u = gu.view(-1, F // 128, 2, 128)[:, :, 0].reshape(-1, F), gu.view(-1, F // 128, 2, 128)[:, :, 1].reshape(-1, F)
            yr[sel] = (torch.nn.functional.silu(g) * u) @ w2_local[e].t()
    ys = torch.empty_like(xs)
    dist.all_to_all_single(ys, yr, sc, rc)
    out = torch.zeros(T * K, x.shape[1], dtype=torch.float32, device=x.device)
    out[order] = ys.float() * w.view(-1)[order][:, None]
    return out.view(T, K, -1).sum(1).to(x.dtype)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=4096, help="tokens per GPU")
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--ffn", type=int, default=14336)
    ap.add_argument("--experts", type=int, default=8)
    ap.add_argument("--top-k", type=int, default=2)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--check", action="store_true")
    args = ap.parse_args()
    info = init_distributed(timeout_s=120.0)
    W, R, dev = info.world, info.rank, info.device
    H, F, E, K = args.hidden, args.ffn, args.experts, args.top_k
    if args.check:
        H, F = 1024, 1536
    T = args.tokens if not args.check else 700 + 37 * R
    E_l = E // W
    local = [expert_weights(R * E_l + e, H, F, dev) for e in range(E_l)]
    w13 = torch.stack([l[0] for l in local])
    w2 = torch.stack([l[1] for l in local])
    moe = EpMoE(info, E, H, F, K, max_tokens=max(T, 1024) + 64)
    g = torch.Generator(device=dev).manual_seed(50 + R)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    router = (torch.randn(H, E, generator=torch.Generator(device=dev).manual_seed(3), device=dev) * 0.05).to(torch.bfloat16)
    idx, w = route(x @ router, K)
    ok_all = True
    recs = []
    if args.check:
        allw = [expert_weights(e, H, F, dev) for e in range(E)]
        ref = experts_reference(x, idx, w, torch.stack([a for a, _ in allw]), torch.stack([b for _, b in allw]), 0)
        for it in range(3):  # repeated calls: epochs, counters and flags are reused
            y = moe.forward(x, idx, w, w13, w2)
            torch.cuda.synchronize()
            rel = float((y.float() - ref).norm() / ref.norm())
            ok = rel < 2e-2 and check_errors(dev) == 0
            ok_all &= ok
            recs.append({"check": "ep_moe", "world": W, "rank": R, "iter": it, "rel_err": rel, "ok": ok})
        # skewed routing: every pair to expert 0's GPU
        idx0 = torch.zeros_like(idx)
        idx0[:, 1] = E - 1
        y0 = moe.forward(x, idx0, w, w13, w2)
        ref0 = experts_reference(x, idx0, w, torch.stack([a for a, _ in allw]), torch.stack([b for _, b in allw]), 0)
        torch.cuda.synchronize()
        rel0 = float((y0.float() - ref0).norm() / ref0.norm())
        ok0 = rel0 < 2e-2 and check_errors(dev) == 0
        ok_all &= ok0
        recs.append({"check": "ep_moe_skewed", "rank": R, "rel_err": rel0, "ok": ok0})
        ok_all = bool(all_reduce_max(0.0 if ok_all else 1.0, info) == 0.0)
    else:
        def timed(fn):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            barrier(info)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.iters):
                fn()
            e1.record()
            torch.cuda.synchronize()
            return all_reduce_max(e0.elapsed_time(e1) / args.iters, info)

        fused = timed(lambda: moe.forward(x, idx, w, w13, w2))
        base = timed(lambda: nccl_layer(x, idx, w, w13, w2, E_l, W, R)) if W > 1 else None
        flops = 2.0 * T * K * (2 * F * H + H * F) * W
        recs.append({"layer": "moe_ep", "world": W, "tokens_per_gpu": T, "hidden": H, "ffn": F, "experts": E,
                     "top_k": K, "fused_ms": fused, "nccl_cublas_ms": base,
                     "fused_tflops_total": flops / fused / 1e9, "speedup": (base / fused) if base else None,
                     "errors": check_errors(dev)})
    if R == 0:
        for r in recs:
            print(json.dumps(r), flush=True)
        if args.check:
            print("EP_CHECK", "ok" if ok_all else "FAILED", flush=True)
    del moe
    shutdown(info)
    if not ok_all:
        sys.exit(1)


if __name__ == "__main__":
    main()
