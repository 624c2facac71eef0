"""Process-group bootstrap: one process per GPU.

Reads RANK / LOCAL_RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT (as set by
``torch.distributed.run``).  NCCL is the backend on GPU; gloo runs the same
host-side logic on CPU.  The reference initialises JAX distributed with a Ray
coordinator instead (src/flare/jax/training/engines/distributed.py:47-94).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class WorldInfo:
    rank: int = 0
    world_size: int = 1
    local_rank: int = 0
    local_world_size: int = 1
    backend: str = "none"

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1

    @property
    def node_rank(self) -> int:
        return self.rank // max(self.local_world_size, 1)


def env_world() -> WorldInfo:
    return WorldInfo(
        rank=int(os.environ.get("RANK", 0)),
        world_size=int(os.environ.get("WORLD_SIZE", 1)),
        local_rank=int(os.environ.get("LOCAL_RANK", 0)),
        local_world_size=int(os.environ.get("LOCAL_WORLD_SIZE", os.environ.get("WORLD_SIZE", 1))),
    )


def init_distributed(backend: str | None = None, timeout_s: float = 120.0) -> WorldInfo:
    """Initialise torch.distributed from the environment (no-op for world size 1)."""
    info = env_world()
    if torch.cuda.is_available():
        torch.cuda.set_device(info.local_rank)
    if info.world_size <= 1:
        return WorldInfo(backend="none")
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29511")
        backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
        kwargs = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kwargs["device_id"] = torch.device("cuda", info.local_rank)
        dist.init_process_group(**kwargs)
    return WorldInfo(info.rank, info.world_size, info.local_rank, info.local_world_size, dist.get_backend())


def barrier() -> None:
    if dist.is_initialized() and dist.get_world_size() > 1:
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def all_gather_object(obj):
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return [obj]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def max_over_ranks(value: float) -> float:
    """Max of a host scalar over ranks (used for device-timed step times)."""
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shutdown() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


__all__ = ["WorldInfo", "all_gather_object", "barrier", "env_world", "init_distributed", "max_over_ranks",
           "shutdown"]
