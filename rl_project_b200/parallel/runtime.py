"""Process-group lifecycle and rank helpers (``src/forgeline/distributed/runtime.py`` contract).

One process per GPU; NCCL on CUDA, gloo on CPU.  Unlike the reference, every
process group is created with an explicit ``timeout`` (``DistributedConfig.timeout_s``)
so a dead or stalled rank turns into an error instead of a hang, and the
rendezvous defaults to 127.0.0.1.
"""

from __future__ import annotations

import datetime
import os
import socket
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from rl_project_b200.core.errors import DistributedConfigError


@dataclass
class DistributedInfo:
    rank: int
    local_rank: int
    world_size: int
    backend: str
    launched: bool


def read_launcher_env() -> DistributedInfo:
    launched = "RANK" in os.environ and "WORLD_SIZE" in os.environ
    return DistributedInfo(rank=int(os.environ.get("RANK", 0)), local_rank=int(os.environ.get("LOCAL_RANK", 0)),
                           world_size=int(os.environ.get("WORLD_SIZE", 1)), backend="", launched=launched)


def select_backend(requested: str = "auto") -> str:
    if requested == "auto":
        return "nccl" if torch.cuda.is_available() else "gloo"
    if requested == "nccl" and not torch.cuda.is_available():
        raise DistributedConfigError("backend=nccl requires CUDA", hint="Use backend=gloo on CPU.")
    return requested


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def init_process_group(backend: str = "auto", *, world_size: Optional[int] = None, rank: Optional[int] = None,
                       init_method: Optional[str] = None, timeout_s: float = 600.0) -> DistributedInfo:
    info = read_launcher_env()
    backend = select_backend(backend)
    if torch.cuda.is_available() and backend == "nccl":
        torch.cuda.set_device(info.local_rank)
    if not dist.is_initialized():
        kw = dict(backend=backend, world_size=world_size if world_size is not None else info.world_size,
                  rank=rank if rank is not None else info.rank, timeout=datetime.timedelta(seconds=timeout_s))
        if init_method is not None:
            kw["init_method"] = init_method
        else:
            if not info.launched:
                os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
                os.environ.setdefault("MASTER_PORT", str(free_port()))
            kw["init_method"] = "env://"
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", info.local_rank)
        dist.init_process_group(**kw)
    return DistributedInfo(rank=dist.get_rank(), local_rank=info.local_rank, world_size=dist.get_world_size(),
                           backend=backend, launched=info.launched)


def destroy_process_group() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


def is_initialized() -> bool:
    return dist.is_initialized()


def is_main_process() -> bool:
    return not dist.is_initialized() or dist.get_rank() == 0


def world_size() -> int:
    return dist.get_world_size() if dist.is_initialized() else 1


def rank() -> int:
    return dist.get_rank() if dist.is_initialized() else 0


def barrier() -> None:
    if dist.is_initialized() and dist.get_world_size() > 1:
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def all_reduce_mean(t: torch.Tensor) -> torch.Tensor:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return t
    out = t.clone()
    dist.all_reduce(out)
    return out / dist.get_world_size()


def validate_topology(world: int, tensor_parallel: int, pipeline_parallel: int, expert_parallel: int = 1) -> int:
    if min(tensor_parallel, pipeline_parallel, expert_parallel) < 1:
        raise DistributedConfigError("parallel degrees must be >= 1")
    if world % (tensor_parallel * pipeline_parallel) != 0:
        raise DistributedConfigError(
            f"world_size {world} is not divisible by tensor_parallel {tensor_parallel} x pipeline_parallel "
            f"{pipeline_parallel}")
    dp = world // (tensor_parallel * pipeline_parallel)
    if expert_parallel > 1 and (dp * tensor_parallel) % expert_parallel != 0:
        raise DistributedConfigError(f"expert_parallel {expert_parallel} must divide dp*tp = {dp * tensor_parallel}")
    return dp
