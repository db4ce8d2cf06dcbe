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
    ab = sub.add_parser("amf-bench", help="cold then warm generation of one prompt through the AMF tiers, "
                                          "with [AMF_*] trace lines and a run summary")
    ab.add_argument("--model", default="tiny128")
    ab.add_argument("--prompt-tokens", type=int, default=2048)
    ab.add_argument("--max-tokens", type=int, default=32)
    ab.add_argument("--warm-runs", type=int, default=3)
    ab.add_argument("--device", default=None)
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


def _cmd_amf_bench(a) -> int:
    """Benchmark mode of the reference's vLLM server (korith_vllm_server.py:52-180): one
    cold run captures the prompt's prefix, the live cache is dropped, warm runs restore it.
    Trace lines go to stderr, the summary JSON to stdout."""
    import numpy as np
    import torch

    from ..config import KorithConfig
    from ..engine.engine import SamplingParams

    dev = a.device or ("cuda" if torch.cuda.is_available() else "cpu")
    kcfg = KorithConfig.from_env()
    kcfg.enable_amf = False  # G1 pool only; the disk store is opted into through KORITH_* variables
    kcfg.vram_cache_gb = kcfg.vram_cache_gb or 1.0
    from .app import build_engine

    eng = build_engine(AxropusConfig.load(None, {"model": a.model, "device": dev}), kcfg)
    eng.trace.enabled = True
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, eng.model.cfg.vocab, a.prompt_tokens).tolist()
    sp = SamplingParams(max_tokens=a.max_tokens)
    runs = []
    for i in range(1 + a.warm_runs):
        if i == 1:
            eng.evict_live_cache()
        r = eng.add_request(prompt, sp, amf_prefix_len=a.prompt_tokens - 1)
        while eng.has_unfinished():
            eng.step()
        if i > 0:
            eng.evict_live_cache()
        runs.append({"run": "cold" if i == 0 else "warm", "tier": r.amf_tier, "ttft_ms": round(r.ttft_ms, 3),
                     "restored_tokens": r.restored_tokens, "restore_ms": round(r.restore_ms, 3)})
    summary = eng.run_summary()
    print(json.dumps({"model": eng.model.cfg.name, "device": str(eng.device), "runs": runs, "summary": summary},
                     indent=2, default=str))
    return 0


def main(argv=None) -> int:
    a = build_parser().parse_args(argv)
    return {"serve": _cmd_serve, "bench": _cmd_bench, "info": _cmd_info, "amf-bench": _cmd_amf_bench}[a.command](a)


if __name__ == "__main__":
    sys.exit(main())
