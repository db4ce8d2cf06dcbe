"""Failure detection and recovery, exercised on the host (no GPU is faulted, trapped or
hung): a rank that dies mid-capture while pinning a pool entry, a dead peer seen by the
process group, a fused-kernel wait timeout turned into an engine error, and a corrupted
AMF blob turned into a miss."""
import os
import socket
import tempfile
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from axropus_deploy_b200.amf.keys import pool_key, pool_key_int
    from axropus_deploy_b200.ops.kvcache import KVCache
    from axropus_deploy_b200.parallel.dist import DistInfo
    from axropus_deploy_b200.parallel.sharded_pool import build_pool, cleanup_shm

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    info = DistInfo(rank, world, rank, world, torch.device("cpu"))
    tag = f"fail_{port}"
    pool = build_pool(info, 2, 2, 64, "fp8", 64, tag)
    cache = KVCache(2, 16, 2, 64, "bf16", "cpu")
    cache.data.normal_()
    p1, p2 = list(range(100, 164)), list(range(500, 564))
    if rank == 1:
        assert pool.capture(pool_key(p1), cache, torch.arange(4, dtype=torch.int32), 64)
        hit = pool.lookup(pool_key(p1))  # pinned by rank 1 (an in-flight restore)
        assert hit is not None
        # a capture that starts and never finishes (the process dies mid-copy)
        shard = pool.owner(pool_key(p2))
        st, slots, _ = pool.dir.begin_insert(shard, pool_key_int(pool_key(p2)), 0, 4, 64, 1, 1, 0.0)
        assert str(st).endswith("OK")
        dist.barrier()
        os._exit(0)  # dies without unpinning, committing or destroying the group
    dist.barrier()  # rank 1 has pinned and half-written by now
    time.sleep(1.0)
    res = {}
    # the process group notices the dead peer on the next collective (error or timeout)
    t0 = time.time()
    try:
        dist.barrier()
        res["pg_error"] = False
    except Exception:
        res["pg_error"] = True
    res["pg_detect_s"] = time.time() - t0
    s1 = pool.owner(pool_key(p1))
    k1 = pool_key_int(pool_key(p1))
    res["pins_before"] = [e["pins"] for e in pool.dir.entries(s1) if e["key"] == k1]
    res["writing_before"] = sum(1 for s in range(world) for e in pool.dir.entries(s) if e["writer"] == 1
                                and e["key"] == pool_key_int(pool_key(p2)))
    res["released"] = int(pool.dir.release_rank(1))
    res["pins_after"] = [e["pins"] for e in pool.dir.entries(s1) if e["key"] == k1]
    res["p1_ready"] = pool.contains(pool_key(p1))
    res["p2_present"] = any(e["key"] == pool_key_int(pool_key(p2)) for s in range(world) for e in pool.dir.entries(s))
    # the freed slots take a new entry
    res["recapture"] = pool.capture(pool_key(p2), cache, torch.arange(4, dtype=torch.int32), 64)
    torch.save(res, os.path.join(out_dir, "r0.pt"))
    cleanup_shm(tag, world, "fp8")
    os._exit(0)


def test_dead_rank_released_and_detected():
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        res = torch.load(os.path.join(d, "r0.pt"))
    assert res["pg_error"] and res["pg_detect_s"] < 30
    assert res["pins_before"] == [1] and res["writing_before"] == 1
    assert res["released"] >= 2
    assert res["pins_after"] == [0] and res["p1_ready"]
    assert not res["p2_present"] and res["recapture"]


def test_kernel_wait_timeout_becomes_engine_error(monkeypatch):
    """A fused kernel that gave up waiting on a peer records a code; the engine raises
    instead of handing out the step's outputs."""
    from axropus_deploy_b200.engine.engine import EngineConfig, LLMEngine
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel
    from axropus_deploy_b200.ops import gemm as gemm_mod

    eng = LLMEngine(LlamaModel(get_config("tiny128"), "cpu", torch.float32), EngineConfig(num_blocks=16))
    flag = torch.zeros(4, dtype=torch.int32)
    monkeypatch.setattr(gemm_mod, "error_flag", lambda dev: flag)
    eng._check_kernel_errors()  # no error recorded
    flag[0] = 43  # e.g. the MoE gate/up producer gave up on a source's arrival flag
    with pytest.raises(RuntimeError, match="error code 43"):
        eng._check_kernel_errors()


def test_corrupted_amf_blob_is_a_miss(tmp_path):
    from axropus_deploy_b200.amf.disk import DiskTier

    tier = DiskTier(str(tmp_path / "amf"), config={"min_tokens": 16})
    assert tier.enabled
    toks = list(range(1, 65))
    pages = torch.randn(4, 2, 2, 2, 16, 64).to(torch.bfloat16)
    assert tier.save(toks, pages, saved_ms=50)
    reason, entry = tier.lookup(toks + [7, 8])
    assert entry is not None
    good = tier.load(entry)
    assert good is not None and torch.equal(good[1], pages)
    kv = [f for f in os.listdir(tmp_path / "amf") if f.endswith(".kv")]
    assert len(kv) == 1
    path = tmp_path / "amf" / kv[0]
    raw = bytearray(path.read_bytes())
    raw[len(raw) // 2] ^= 0xFF  # one flipped byte in the payload
    path.write_bytes(bytes(raw))
    assert tier.load(entry) is None  # checksum mismatch: fail closed, the caller prefills
    path.write_bytes(bytes(raw[: len(raw) // 3]))  # truncated blob
    assert tier.load(entry) is None
