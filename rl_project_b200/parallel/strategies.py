"""Distributed strategies behind one interface (``DistributedStrategy`` protocol,
``src/forgeline/distributed/strategies.py:17-218`` names):
single, ddp, fsdp, zero2, deepspeed, tensor_parallel, pipeline_parallel,
expert_parallel, hybrid (3-D mesh).

Each strategy validates on CPU; ``setup`` only creates a process group when
launched (or when a 1-process group is explicitly allowed).
"""

from __future__ import annotations

from typing import Any, Optional

import torch
import torch.nn as nn

from rl_project_b200.core.config import DistributedConfig
from rl_project_b200.core.errors import DistributedConfigError, OptionalDependencyError
from rl_project_b200.parallel import runtime as rt


class _OneProcess:
    """Topology of a run without a process group: a single rank."""

    @staticmethod
    def rank() -> int:
        return 0

    @staticmethod
    def size() -> int:
        return 1

    @staticmethod
    def sync() -> None:
        return None

    @staticmethod
    def leave() -> None:
        return None


class _DefaultGroup:
    """Topology of torch.distributed's default process group, read live (answers like one rank until the
    group exists)."""

    rank = staticmethod(rt.rank)
    size = staticmethod(rt.world_size)
    sync = staticmethod(rt.barrier)
    leave = staticmethod(rt.destroy_process_group)


class SingleProcessStrategy:
    """Base of every strategy: rank queries go to its topology object (one process here, the default
    process group for the distributed strategies); subclasses add ``setup`` and the model wrapper."""

    name = "single"
    topology = _OneProcess

    def __init__(self, cfg: Optional[DistributedConfig] = None):
        self.cfg = cfg or DistributedConfig()
        self.monitor = None

    def setup(self) -> None:
        return None

    def wrap_model(self, model: nn.Module) -> nn.Module:
        return model

    def unwrap_model(self, model: nn.Module) -> nn.Module:
        return model

    def rank(self) -> int:
        return self.topology.rank()

    def world_size(self) -> int:
        return self.topology.size()

    def is_main_process(self) -> bool:
        return self.rank() == 0

    def barrier(self) -> None:
        self.topology.sync()

    def check_health(self) -> None:
        """Raise DistributedTimeoutError if a peer rank stopped beating (called between steps)."""
        if self.monitor is not None:
            self.monitor.check()

    def teardown(self) -> None:
        if self.monitor is not None:
            self.monitor.stop("teardown")
            self.monitor = None
        self.topology.leave()


class _ProcessGroupStrategy(SingleProcessStrategy):
    """Joins (or creates, when not launched and a one-process group is allowed) the default process group and
    starts the store heartbeat when the config asks for one."""

    topology = _DefaultGroup

    def __init__(self, cfg: DistributedConfig, allow_single_process: bool = True):
        super().__init__(cfg)
        self.allow_single_process = allow_single_process
        self.info: Optional[rt.DistributedInfo] = None

    def setup(self) -> None:
        if not (rt.read_launcher_env().launched or self.allow_single_process):
            raise DistributedConfigError(f"{self.name} strategy requires a torchrun launch (RANK/WORLD_SIZE not set)")
        self.info = rt.init_process_group(self.cfg.backend, timeout_s=self.cfg.timeout_s)
        self.start_health_monitor()

    def start_health_monitor(self) -> None:
        from rl_project_b200.parallel.health import monitor_for_process_group

        every = float(getattr(self.cfg, "heartbeat_interval_s", 0.0) or 0.0)
        limit = float(getattr(self.cfg, "heartbeat_timeout_s", 60.0))
        self.monitor = monitor_for_process_group(every, limit) if every > 0 else None

    def unwrap_model(self, model: nn.Module) -> nn.Module:
        return getattr(model, "module", model)


class DDPStrategy(_ProcessGroupStrategy):
    """Replicated parameters; bucketed gradient all-reduce after accumulation (Trainer-driven)."""

    name = "ddp"

    def wrap_model(self, model: nn.Module) -> nn.Module:
        if not rt.is_initialized():
            raise DistributedConfigError("call setup() before wrap_model()")
        if rt.world_size() == 1:
            return model
        from torch.nn.parallel import DistributedDataParallel as DDP

        ids = [self.info.local_rank] if self.info and torch.cuda.is_available() else None
        return DDP(model, device_ids=ids, find_unused_parameters=True)


class DeepSpeedStrategy(_ProcessGroupStrategy):
    name = "deepspeed"

    def __init__(self, cfg: DistributedConfig):
        super().__init__(cfg)
        self.config_path = cfg.deepspeed_config

    @staticmethod
    def load_config(path: str) -> dict:
        import json
        from pathlib import Path

        p = Path(path)
        if not p.exists():
            raise DistributedConfigError(f"deepspeed config not found: {path}")
        data = json.loads(p.read_text())
        if "zero_optimization" not in data:
            raise DistributedConfigError("deepspeed config must contain zero_optimization")
        return data

    def initialize(self, model: nn.Module, optimizer=None) -> Any:
        try:
            import deepspeed
        except ImportError as exc:
            raise OptionalDependencyError("deepspeed is not installed",
                                          hint="Use strategy=zero2 (the native ZeRO-2) instead.") from exc
        engine, _, _, _ = deepspeed.initialize(model=model, optimizer=optimizer, config=self.load_config(self.config_path),
                                               model_parameters=[p for p in model.parameters() if p.requires_grad])
        return engine

    def wrap_model(self, model: nn.Module) -> nn.Module:
        return self.initialize(model)


# strategy name -> (module, class, constructor keywords); the heavier strategies import on first use
_LAZY = {
    "fsdp": ("rl_project_b200.parallel.fsdp", "FSDPStrategy", {}),
    "zero2": ("rl_project_b200.parallel.fsdp", "FSDPStrategy", {"reshard_params": False, "name": "zero2"}),
    "tensor_parallel": ("rl_project_b200.parallel.mesh_strategies", "MeshStrategy", {"name": "tensor_parallel"}),
    "pipeline_parallel": ("rl_project_b200.parallel.mesh_strategies", "MeshStrategy", {"name": "pipeline_parallel"}),
    "hybrid": ("rl_project_b200.parallel.mesh_strategies", "MeshStrategy", {"name": "hybrid"}),
    "expert_parallel": ("rl_project_b200.parallel.expert", "ExpertParallelStrategy", {}),
}


def _lazy(name: str):
    module, cls, kw = _LAZY[name]

    def make(cfg: DistributedConfig):
        import importlib

        return getattr(importlib.import_module(module), cls)(cfg, **kw)

    return make


STRATEGIES = {"single": SingleProcessStrategy, "ddp": DDPStrategy, "deepspeed": DeepSpeedStrategy,
              **{name: _lazy(name) for name in _LAZY}}


def build_strategy(cfg: DistributedConfig):
    cfg.validate()
    if cfg.strategy not in STRATEGIES:
        raise DistributedConfigError(f"unknown strategy {cfg.strategy!r}")
    return STRATEGIES[cfg.strategy](cfg)


def validate_distributed_config(cfg: DistributedConfig, world_size: Optional[int] = None) -> dict:
    """CPU-only check of a distributed config: returns the implied topology or raises
    ``DistributedConfigError`` (``src/forgeline/distributed/strategies.py:221-232`` contract,
    extended with the expert-parallel degree)."""
    from rl_project_b200.parallel import runtime as rt

    cfg.validate()
    ws = world_size if world_size is not None else rt.read_launcher_env().world_size
    dp = rt.validate_topology(ws, cfg.tensor_parallel_size, cfg.pipeline_parallel_size, cfg.expert_parallel_size)
    needs = {"tensor_parallel": cfg.tensor_parallel_size, "pipeline_parallel": cfg.pipeline_parallel_size,
             "expert_parallel": cfg.expert_parallel_size}
    if cfg.strategy in needs and needs[cfg.strategy] == 1:
        raise DistributedConfigError(f"{cfg.strategy} strategy needs {cfg.strategy}_size > 1")
    if cfg.strategy == "deepspeed":
        DeepSpeedStrategy.load_config(cfg.deepspeed_config)
    return {"world_size": ws, "tensor_parallel": cfg.tensor_parallel_size,
            "pipeline_parallel": cfg.pipeline_parallel_size, "expert_parallel": cfg.expert_parallel_size,
            "data_parallel": dp}
