"""Orchestration settings, importable without Ray.

``RayConfig`` carries the manifest keys of ``src/forgeline/orchestration/config.py`` and is validated
against the ``_RULES`` table; ``validate_orchestration`` checks an ``orchestration`` mapping without
importing Ray (the check of ``src/forgeline/orchestration/__init__.py``).
"""

from __future__ import annotations

import dataclasses
import importlib.util
from dataclasses import dataclass
from typing import Any, Dict, Mapping, Optional

from rl_project_b200.core.errors import ConfigError

PLACEMENT_STRATEGIES = ("PACK", "SPREAD", "STRICT_PACK", "STRICT_SPREAD")
ORCHESTRATION_TYPES = ("local", "ray")


@dataclass
class RayConfig:
    address: Optional[str] = None
    num_cpus: Optional[int] = None
    num_gpus: Optional[int] = None
    rollout_workers: int = 0
    reward_workers: int = 0
    cpus_per_worker: float = 1.0
    gpus_per_worker: float = 0.0
    memory_per_worker_mb: Optional[int] = None
    placement_strategy: Optional[str] = None
    placement_timeout_s: float = 60.0
    max_restarts: int = 1
    max_call_retries: int = 2
    task_timeout_s: Optional[float] = None
    worker_torch_threads: int = 1
    namespace: str = "forgeline"
    backend: str = "ray"  # "ray" actors, or "threads": in-process workers (single node, tests)

    def validate(self) -> None:
        for broken, message in _RULES:
            if broken(self):
                raise ConfigError(message)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> "RayConfig":
        names = {f.name for f in dataclasses.fields(cls)}
        bad = sorted(set(data) - names)
        if bad:
            raise ConfigError(f"unknown orchestration keys: {bad}")
        cfg = cls(**dict(data))
        cfg.validate()
        return cfg

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


# (condition that makes a config invalid, message), checked in order
_RULES = (
    (lambda c: c.backend not in ("ray", "threads"), "orchestration.backend must be 'ray' or 'threads'"),
    (lambda c: c.address is not None and (c.num_cpus is not None or c.num_gpus is not None),
     "orchestration.num_cpus/num_gpus apply only when Ray is started locally (address unset)"),
    (lambda c: min(c.rollout_workers, c.reward_workers) < 0, "orchestration worker counts must be >= 0"),
    (lambda c: min(c.cpus_per_worker, c.gpus_per_worker) < 0, "orchestration per-worker resources must be >= 0"),
    (lambda c: c.placement_strategy is not None and c.placement_strategy not in PLACEMENT_STRATEGIES,
     f"placement_strategy must be one of {PLACEMENT_STRATEGIES}"),
    (lambda c: c.max_restarts < -1 or c.max_call_retries < 0, "max_restarts must be >= -1 and max_call_retries >= 0"),
)


def ray_available() -> bool:
    return importlib.util.find_spec("ray") is not None


def validate_orchestration(config: Mapping[str, Any]) -> None:
    if not config:
        return
    kind = config.get("type", "local")
    if kind not in ORCHESTRATION_TYPES:
        raise ConfigError(f"orchestration.type must be one of {ORCHESTRATION_TYPES}, got {kind!r}")
    if kind == "ray":
        RayConfig.from_dict({k: v for k, v in config.items() if k != "type"})


def orchestration_summary(config: Mapping[str, Any]) -> Dict[str, Any]:
    return {"type": (config or {}).get("type", "local"), "ray_installed": ray_available()}
