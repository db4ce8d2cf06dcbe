"""BASELINE config 1 -- CPU plumbing, no GPU.

Tiny Llama-shaped KV (2 layers, 4 KV heads, head_dim 64, 16-token pages, bf16 values
~N(0,1) from seed 0). A 512-token prefix of uniform random token ids in [0, 32000) is
captured into the G1 pool stored raw, FP8-e4m3 per-block scaled and INT4 group-64
asymmetric, then restored into a freshly allocated paged cache with a shuffled block
table. Reports bit-exactness (raw), max-abs error (FP8 / INT4) and an on-disk AMF
store reload (AMFK blob through the native store, reloaded by a fresh store).
"""
import json
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from axropus_deploy_b200.amf import DiskTier, G1Pool  # noqa: E402
from axropus_deploy_b200.amf.keys import AmfContext, pool_key  # noqa: E402
from axropus_deploy_b200.amf.pool import DenseStore  # noqa: E402
from axropus_deploy_b200.ops import KVCache, page_transfer  # noqa: E402

L, H, D, PAGE, T = 2, 4, 64, 16, 512


def run() -> dict:
    g = torch.Generator().manual_seed(0)
    tokens = torch.randint(0, 32000, (T,), generator=g).numpy().astype(np.int32)
    n = T // PAGE
    src = KVCache(L, 64, H, D, "bf16", "cpu")
    src_blocks = torch.randperm(64, generator=g)[:n].to(torch.int32)
    src.write_units(src_blocks, torch.randn(n, L, 2, H, PAGE, D, generator=g).to(torch.bfloat16).float())
    orig = src.read_units(src_blocks)
    key = pool_key(tokens)
    report = {"prefix_tokens": T, "pages": n, "key": key}
    for fmt in ("raw", "fp8", "int4"):
        pool = G1Pool(L, H, D, fmt, slots_per_shard=64, device="cpu")
        assert pool.capture(key, src, src_blocks, T)
        hit = pool.lookup(key)
        dst = KVCache(L, 96, H, D, "bf16", "cpu")
        dst_blocks = torch.randperm(96, generator=g)[:n].to(torch.int32)  # shuffled block table
        pool.restore(hit, dst, dst_blocks)
        pool.release(hit)
        back = dst.read_units(dst_blocks)
        if fmt == "raw":
            report["raw_bit_exact"] = bool(torch.equal(dst.data[:, :, dst_blocks.long()], src.data[:, :, src_blocks.long()]))
        else:
            report[f"{fmt}_max_abs_err"] = float((back - orig).abs().max())
            report[f"{fmt}_rel_err"] = float((back - orig).norm() / orig.norm())
        report[f"{fmt}_bytes"] = pool.used_bytes()
    with tempfile.TemporaryDirectory() as d:
        ctx = AmfContext(model_hash=0x1234, n_ctx=4096, kv_version=1)
        disk = DiskTier(d, ctx, {"min_tokens": 64})
        dense = DenseStore(torch.empty(n, L, 2, H, PAGE, D, dtype=torch.bfloat16))
        page_transfer(src, src_blocks, dense, torch.arange(n, dtype=torch.int32))
        assert disk.save(tokens, dense.t, saved_ms=50)
        disk.store.shutdown()
        disk2 = DiskTier(d, ctx, {"min_tokens": 64})
        reason, entry = disk2.lookup(np.concatenate([tokens, tokens[:40]]))
        hdr, pages = disk2.load(entry)
        report["disk_lookup"] = reason
        report["disk_reload_bit_exact"] = bool(torch.equal(pages, dense.t))
        report["amfk_header"] = {"n_layers": hdr.n_layers, "n_tokens": hdr.n_tokens, "n_kv_heads": hdr.n_kv_heads,
                                 "head_dim": hdr.head_dim, "dtype": hdr.dtype}
    return report


if __name__ == "__main__":
    print(json.dumps(run(), indent=1))
