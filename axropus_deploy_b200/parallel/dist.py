"""Process-group plumbing: one process per GPU, NCCL over NVLink for control
collectives (gloo on CPU-only ranks), short timeouts so a rank that waits on a dead
peer ends with an error instead of hanging."""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class DistInfo:
    rank: int = 0
    world: int = 1
    local_rank: int = 0
    local_world: int = 1
    device: torch.device = torch.device("cpu")

    @property
    def is_dist(self) -> bool:
        return self.world > 1


def init_distributed(backend: Optional[str] = None, timeout_s: float = 120.0) -> DistInfo:
    """Initialise from RANK / WORLD_SIZE / LOCAL_RANK / MASTER_* (torchrun's env).
    Without them this is a single-process run."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    cuda = torch.cuda.is_available()
    if cuda:
        torch.cuda.set_device(local_rank % torch.cuda.device_count())
        device = torch.device("cuda", torch.cuda.current_device())
    else:
        device = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        be = backend or ("nccl" if cuda else "gloo")
        kw = {"device_id": device} if be == "nccl" else {}
        dist.init_process_group(be, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return DistInfo(rank, world, local_rank, local_world, device)


def barrier(info: DistInfo) -> None:
    if info.is_dist:
        if info.device.type == "cuda":
            dist.barrier(device_ids=[info.device.index])
        else:
            dist.barrier()


def all_reduce_max(x: float, info: DistInfo) -> float:
    if not info.is_dist:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=info.device if info.device.type == "cuda" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_reduce_min(x: float, info: DistInfo) -> float:
    if not info.is_dist:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=info.device if info.device.type == "cuda" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return float(t.item())


def all_reduce_sum(x: float, info: DistInfo) -> float:
    if not info.is_dist:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=info.device if info.device.type == "cuda" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def all_gather_object(obj, info: DistInfo) -> list:
    if not info.is_dist:
        return [obj]
    out = [None] * info.world
    dist.all_gather_object(out, obj)
    return out


def job_tag() -> str:
    """A name shared by every rank of this job (used for shared-memory objects)."""
    return os.environ.get("AXR_JOB_TAG") or f"axr_{os.environ.get('MASTER_PORT', '0')}_{os.getppid() if 'RANK' in os.environ else os.getpid()}"


def shutdown(info: DistInfo) -> None:
    if info.is_dist and dist.is_initialized():
        dist.destroy_process_group()
