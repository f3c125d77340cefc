"""Run lifecycle: the ``Stage`` names of a post-training pipeline and ``RunContext``, the per-run bundle of
manifest, seed, device placement, compute dtype, output directory and metrics sink (the contract of
``src/forgeline/core/lifecycle.py:19-77``).

``RunContext.create`` validates the manifest, seeds every RNG, places the run (device from the manifest or an
override; the compute dtype the device supports), opens the metrics sink in the output directory and logs one
``run_context`` line.  A context is also a context manager that closes its sink on exit.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from enum import Enum
from pathlib import Path
from typing import Any, Dict, Optional, Tuple

import torch

from rl_project_b200.core.config import ExperimentManifest
from rl_project_b200.core.runtime import resolve_device, resolve_dtype, seed_everything
from rl_project_b200.observability.logging import get_logger
from rl_project_b200.observability.metrics import MetricsSink, build_metrics_sink

# pipeline stages, in the order a full run visits them
Stage = Enum("Stage", [(n.upper(), n) for n in ("data", "pretrain", "sft", "reward_model", "preference", "rl",
                                                 "evaluation", "export", "serving", "deployment")], type=str)


def _placement(manifest: ExperimentManifest, distributed: bool,
               device_override: Optional[str]) -> Tuple[torch.device, torch.dtype]:
    device = resolve_device(device_override or manifest.trainer.device, distributed=distributed)
    return device, resolve_dtype(manifest.trainer.precision.dtype, device)


@dataclass
class RunContext:
    manifest: ExperimentManifest
    device: torch.device
    dtype: torch.dtype
    output_dir: Path
    metrics: MetricsSink
    seed: int
    started_at: float = field(default_factory=time.time)
    extra: Dict[str, Any] = field(default_factory=dict)

    @classmethod
    def create(cls, manifest: ExperimentManifest, *, metrics_backend: str = "local", distributed: bool = False,
               device_override: Optional[str] = None) -> "RunContext":
        manifest.validate()
        seed_everything(manifest.trainer.seed)
        device, dtype = _placement(manifest, distributed, device_override)
        root = Path(manifest.output_dir)
        root.mkdir(parents=True, exist_ok=True)
        ctx = cls(manifest=manifest, device=device, dtype=dtype, output_dir=root, seed=manifest.trainer.seed,
                  metrics=build_metrics_sink(metrics_backend, output_dir=root, run_name=manifest.name,
                                             config=manifest.to_dict()))
        get_logger("run").info("run_context", name=manifest.name, algorithm=manifest.algorithm, device=str(device),
                               dtype=str(dtype), seed=ctx.seed, output_dir=str(root))
        return ctx

    @property
    def logger(self):
        return get_logger(self.manifest.algorithm)

    def elapsed(self) -> float:
        return time.time() - self.started_at

    def close(self) -> None:
        self.metrics.close()

    def __enter__(self) -> "RunContext":
        return self

    def __exit__(self, *exc: Any) -> None:
        self.close()
