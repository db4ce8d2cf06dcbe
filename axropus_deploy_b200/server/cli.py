"""``axropus`` command line (``python -m axropus_deploy_b200``): serve, bench, info
(reference: axropus/cli.py:34-143)."""
from __future__ import annotations

import argparse
import json
import logging
import sys
import time
from pathlib import Path

from ..config import AxropusConfig

VERSION = "0.1.0"


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="axropus", description="B200-native AMF KV materialisation and serving")
    p.add_argument("--version", action="version", version=f"axropus_deploy_b200 {VERSION}")
    sub = p.add_subparsers(dest="command", required=True)
    s = sub.add_parser("serve", help="run the HTTP server")
    for a in ("--model", "--host", "--config", "--log-level", "--api-key"):
        s.add_argument(a, default=None)
    s.add_argument("--port", type=int, default=None)
    b = sub.add_parser("bench", help="codec sweep + kernel microbenchmarks")
    b.add_argument("--config", default=None)
    b.add_argument("--output", default=None)
    b.add_argument("--quick", action="store_true")
    sub.add_parser("info", help="print system information")
    return p


def _cmd_serve(a) -> int:
    overrides = {k: v for k, v in (("model", a.model), ("host", a.host), ("port", a.port),
                                   ("log_level", a.log_level), ("api_key", a.api_key)) if v}
    cfg = AxropusConfig.load(a.config, overrides)
    logging.basicConfig(level=getattr(logging, cfg.log_level.upper(), logging.INFO))
    logging.getLogger("axropus").info("config:\n%s", cfg.summary())
    import uvicorn

    from .app import create_app

    uvicorn.run(create_app(cfg), host=cfg.host, port=cfg.port, log_level=cfg.log_level.lower())
    return 0


def codec_sweep(quick: bool = False) -> dict:
    import torch

    from ..codecs import get_codec, list_codecs

    torch.manual_seed(0)
    x = torch.randn(2, 64 if quick else 256, 8, 128)
    out = {}
    for f in list_codecs():
        c = get_codec(f)
        t0 = time.perf_counter()
        blob = c.compress(x)
        y = c.decompress_to(blob, torch.float32)
        out[f] = {"rel_err": float((y - x).norm() / x.norm()), "ratio": blob.nbytes() / (x.numel() * 2),
                  "ms": (time.perf_counter() - t0) * 1e3}
    return out


def kernel_microbench(quick: bool = False) -> dict:
    import torch

    if not torch.cuda.is_available():
        return {"skipped": "no CUDA device"}
    from ..ops import KVCache, decode_attention

    res = {}
    for T in ([1024, 4096] if quick else [1024, 4096, 16384, 65536]):
        for fmt in ("bf16", "fp8", "int4"):
            pages = T // 16
            cache = KVCache(1, 8 * pages, 8, 128, fmt, "cuda")
            bt = torch.arange(8 * pages, dtype=torch.int32, device="cuda").view(8, pages)
            sl = torch.full((8,), T, dtype=torch.int32, device="cuda")
            q = torch.randn(8, 32, 128, device="cuda").to(torch.bfloat16)
            for _ in range(3):
                decode_attention(q, cache, 0, bt, sl, max_seq_len=T)
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            for _ in range(10):
                decode_attention(q, cache, 0, bt, sl, max_seq_len=T)
            e1.record()
            e1.synchronize()
            res[f"decode_{fmt}_T{T}_B8_us"] = e0.elapsed_time(e1) / 10 * 1e3
    return res


def _cmd_bench(a) -> int:
    res = {"version": VERSION, "codec_sweep": codec_sweep(a.quick), "kernel_microbench": kernel_microbench(a.quick)}
    text = json.dumps(res, indent=2)
    if a.output:
        Path(a.output).write_text(text)
    else:
        print(text)
    return 0


def _cmd_info(a) -> int:
    import torch

    info = {"version": VERSION, "torch": torch.__version__, "cuda": torch.version.cuda,
            "cuda_available": torch.cuda.is_available()}
    if torch.cuda.is_available():
        p = torch.cuda.get_device_properties(0)
        info.update(device=p.name, sm=f"{p.major}{p.minor}", sms=p.multi_processor_count,
                    memory_gb=round(p.total_memory / 2 ** 30, 1))
    try:
        from ..ops._ext import ext_path

        info["kernels"] = ext_path()
    except Exception as exc:
        info["kernels"] = f"not built: {exc}"
    print(json.dumps(info, indent=2))
    return 0


def main(argv=None) -> int:
    a = build_parser().parse_args(argv)
    return {"serve": _cmd_serve, "bench": _cmd_bench, "info": _cmd_info}[a.command](a)


if __name__ == "__main__":
    sys.exit(main())
