"""One-shot peer all-reduce (csrc/kernels/allreduce.cu) vs NCCL all_reduce at decode sizes.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        benchmarks/allreduce.py [--check]

Checks the sum against NCCL (several sizes, repeated calls, and calls replayed from a
captured CUDA graph), then times both (CUDA events, max over ranks). Rank 0 prints JSON
lines and ``AR_CHECK ok``.
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
from axropus_deploy_b200.parallel.tp import PeerAllReduce  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--check", action="store_true")
    ap.add_argument("--iters", type=int, default=200)
    args = ap.parse_args()
    info = init_distributed(timeout_s=120.0)
    dev, R = info.device, info.rank
    ar = PeerAllReduce(info, 1 << 20)
    ok = True
    g = torch.Generator(device=dev).manual_seed(10 + R)
    for n in (8, 16 * 8192, 64 * 8192, 1 << 20):
        for _ in range(3):
            x = torch.randn(n, generator=g, device=dev).to(torch.bfloat16)
            ref = x.float().clone()
            dist.all_reduce(ref)
            y = ar(x.clone())
            torch.cuda.synchronize()
            ok &= bool(torch.allclose(y.float(), ref, atol=5e-2, rtol=2e-2))
    # captured in a CUDA graph: three calls per replay, two replays
    xs = [torch.randn(16 * 8192, generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]
    outs = [torch.empty_like(x) for x in xs]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for x, o in zip(xs, outs):
            ar(x, o)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for x, o in zip(xs, outs):
            ar(x, o)
    for rep in range(2):
        for x in xs:
            x.normal_(generator=g)
        graph.replay()
        torch.cuda.synchronize()
        for x, o in zip(xs, outs):
            ref = x.float().clone()
            dist.all_reduce(ref)
            ok &= bool(torch.allclose(o.float(), ref, atol=5e-2, rtol=2e-2))
    ok &= check_errors(dev) == 0
    ok = all_reduce_max(0.0 if ok else 1.0, info) == 0.0
    recs = []
    if not args.check:
        for rows in (1, 16, 64):
            x = torch.randn(rows * 8192, device=dev).to(torch.bfloat16)

            def timed(fn):
                for _ in range(10):
                    fn()
                torch.cuda.synchronize()
                barrier(info)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(args.iters):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                return all_reduce_max(e0.elapsed_time(e1) / args.iters * 1e3, info)

            recs.append({"bytes": x.numel() * 2, "world": info.world, "peer_us": timed(lambda: ar(x)),
                         "nccl_us": timed(lambda: dist.all_reduce(x))})
    del graph
    if R == 0:
        for r in recs:
            print(json.dumps(r), flush=True)
        print("AR_CHECK", "ok" if ok else "FAILED", flush=True)
    shutdown(info)
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
