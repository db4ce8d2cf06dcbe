"""Expert-parallel Mixtral-style model on CPU ranks (gloo, world 2): each rank serves its
own requests (data-parallel attention) while the MoE layers run over both ranks' experts
in lockstep (an idle rank takes part with empty forwards). Every rank must produce the
greedy tokens of a single-process model holding all experts."""
import os
import socket
import tempfile

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


def _prompts(rank):
    g = torch.Generator().manual_seed(11 + rank)
    lens = (150, 40, 90) if rank == 0 else (33,)  # rank 1 runs out of work early
    return [torch.randint(0, 32000, (n,), generator=g).tolist() for n in lens]


def _full():
    return LlamaModel(get_config("tiny-moe"), "cpu", torch.float32, seed=4, init_std=0.05)


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist

    from axropus_deploy_b200.parallel.dist import DistInfo

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _full()
        info = DistInfo(rank, world, rank, world, torch.device("cpu"))
        m = LlamaModel(get_config("tiny-moe"), "cpu", torch.float32, seed=4, init_std=0.05, ep_info=info)
        E_l = m.cfg.num_experts // world
        for lw, lf in zip(m.layers, full.layers):
            lw.w13 = lf.w13[rank * E_l:(rank + 1) * E_l].clone()
            lw.w2 = lf.w2[rank * E_l:(rank + 1) * E_l].clone()
        assert m.ep is not None and m.expert0 == rank * E_l
        eng = LLMEngine(m, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512, lockstep=True))
        reqs = [eng.add_request(p, SamplingParams(max_tokens=5)) for p in _prompts(rank)]
        steps = 0
        while True:
            flag = torch.tensor([1 if eng.has_unfinished() else 0])
            dist.all_reduce(flag, op=dist.ReduceOp.MAX)
            if int(flag) == 0:
                break
            eng.step()
            steps += 1
        torch.save({"outs": [r.output for r in reqs], "steps": steps}, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_ep_lockstep_matches_full_model():
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _port(), d), nprocs=2, join=True)
        got = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(2)]
    full = _full()
    for rank in range(2):
        ref = LLMEngine(full, EngineConfig(num_blocks=128, max_batch=4, max_model_len=512)).generate(
            _prompts(rank), SamplingParams(max_tokens=5))
        assert got[rank]["outs"] == ref
    assert got[0]["steps"] == got[1]["steps"]
