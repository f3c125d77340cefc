"""Process-group life cycle and rank queries (the functions of ``src/forgeline/distributed/runtime.py``).

One process per GPU: NCCL on CUDA (the process group is bound to the rank's device, so communicators are
created eagerly), gloo on CPU.  Every group gets an explicit timeout (``DistributedConfig.timeout_s``), so a
dead or stalled rank surfaces as an error rather than a hang, and a rendezvous that no launcher set up
defaults to 127.0.0.1 on a free port.
"""

from __future__ import annotations

import datetime
import os
import socket
from dataclasses import dataclass
from typing import Any, Dict, Optional

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

    @classmethod
    def from_env(cls, backend: str = "") -> "DistributedInfo":
        env = os.environ
        return cls(rank=int(env.get("RANK", 0)), local_rank=int(env.get("LOCAL_RANK", 0)),
                   world_size=int(env.get("WORLD_SIZE", 1)), backend=backend,
                   launched="RANK" in env and "WORLD_SIZE" in env)


def read_launcher_env() -> DistributedInfo:
    """What a launcher (``torchrun`` and the like) exported for this process."""
    return DistributedInfo.from_env()


def select_backend(requested: str = "auto") -> str:
    cuda = torch.cuda.is_available()
    if requested == "auto":
        return "nccl" if cuda else "gloo"
    if requested == "nccl" and not cuda:
        raise DistributedConfigError("backend=nccl requires CUDA", hint="Use backend=gloo on CPU.")
    return requested


def free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def _init_kwargs(info: DistributedInfo, backend: str, world_size: Optional[int], rank: Optional[int],
                 init_method: Optional[str], timeout_s: float) -> Dict[str, Any]:
    if init_method is None and not info.launched:  # a single process started by hand
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(free_port()))
    kw: Dict[str, Any] = {"backend": backend, "init_method": init_method or "env://",
                          "world_size": info.world_size if world_size is None else world_size,
                          "rank": info.rank if rank is None else rank,
                          "timeout": datetime.timedelta(seconds=timeout_s)}
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", info.local_rank)
    return kw


def init_process_group(backend: str = "auto", *, world_size: Optional[int] = None, rank: Optional[int] = None,
                       init_method: Optional[str] = None, timeout_s: float = 600.0) -> DistributedInfo:
    info = read_launcher_env()
    backend = select_backend(backend)
    if backend == "nccl":
        torch.cuda.set_device(info.local_rank)
    if not dist.is_initialized():
        dist.init_process_group(**_init_kwargs(info, backend, world_size, rank, init_method, timeout_s))
    return DistributedInfo(dist.get_rank(), info.local_rank, dist.get_world_size(), backend, info.launched)


def destroy_process_group() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()


def is_initialized() -> bool:
    return dist.is_initialized()


def world_size() -> int:
    return dist.get_world_size() if dist.is_initialized() else 1


def rank() -> int:
    return dist.get_rank() if dist.is_initialized() else 0


def is_main_process() -> bool:
    return rank() == 0


def barrier() -> None:
    if world_size() <= 1:
        return
    if dist.get_backend() == "nccl":
        dist.barrier(device_ids=[torch.cuda.current_device()])
    else:
        dist.barrier()


def all_reduce_mean(t: torch.Tensor) -> torch.Tensor:
    """Mean over ranks (a copy; ``t`` is untouched).  NCCL averages in the collective itself."""
    if world_size() == 1:
        return t
    out = t.clone()
    if dist.get_backend() == "nccl":
        dist.all_reduce(out, op=dist.ReduceOp.AVG)
        return out
    dist.all_reduce(out)
    return out / world_size()


def validate_topology(world: int, tensor_parallel: int, pipeline_parallel: int, expert_parallel: int = 1) -> int:
    """The data-parallel degree ``world / (tp * pp)``; expert parallelism must divide ``dp * tp``."""
    if min(tensor_parallel, pipeline_parallel, expert_parallel) < 1:
        raise DistributedConfigError("parallel degrees must be >= 1")
    model_parallel = tensor_parallel * pipeline_parallel
    if world % model_parallel:
        raise DistributedConfigError(f"world_size {world} is not divisible by tensor_parallel {tensor_parallel} x "
                                     f"pipeline_parallel {pipeline_parallel}")
    dp = world // model_parallel
    if expert_parallel > 1 and (dp * tensor_parallel) % expert_parallel:
        raise DistributedConfigError(f"expert_parallel {expert_parallel} must divide dp*tp = {dp * tensor_parallel}")
    return dp
