"""Tensor-parallel Llama on CPU ranks (gloo, world 2): the sharded model must produce the
dense model's greedy tokens, through both the sequence-parallel (all-gather / reduce-
scatter) prefill layout and the replicated decode layout, and TP ranks must agree on
AMF hits."""
import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from axropus_deploy_b200.engine.engine import EngineConfig, LLMEngine, SamplingParams
from axropus_deploy_b200.models.config import get_config
from axropus_deploy_b200.models.llama import LlamaModel


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _prompts():
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, 32000, (n,), generator=g).tolist() for n in (300, 77, 260)]


def _worker(rank, world, port, out_dir, sp_min):
    import torch.distributed as dist

    from axropus_deploy_b200.models.llama_tp import TpLlamaModel
    from axropus_deploy_b200.parallel.dist import DistInfo

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        dense = LlamaModel(get_config("tiny128"), "cpu", torch.float32, seed=3, init_std=0.05)
        info = DistInfo(rank, world, rank, world, torch.device("cpu"))
        model = TpLlamaModel(dense.cfg, info, dtype=torch.float32, dense=dense, max_tokens=1024, sp_min_tokens=sp_min)
        eng = LLMEngine(model, EngineConfig(num_blocks=256, max_batch=8, max_model_len=1024))
        outs = eng.generate(_prompts(), SamplingParams(max_tokens=6))
        assert eng.cache.num_kv_heads == 1
        agreed = model.agree_min(10 + rank)
        if rank == 0:
            torch.save({"outs": outs, "agreed": agreed}, os.path.join(out_dir, "r0.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("sp_min", [0, 100000])
def test_tp_matches_dense(sp_min):
    dense = LlamaModel(get_config("tiny128"), "cpu", torch.float32, seed=3, init_std=0.05)
    ref = LLMEngine(dense, EngineConfig(num_blocks=256, max_batch=8, max_model_len=1024)).generate(
        _prompts(), SamplingParams(max_tokens=6))
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _port(), d, sp_min), nprocs=2, join=True)
        got = torch.load(os.path.join(d, "r0.pt"))
    assert got["agreed"] == 10
    assert got["outs"] == ref
