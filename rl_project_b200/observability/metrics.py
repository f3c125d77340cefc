"""Metrics sinks (memory, no-op, local JSONL, W&B, TensorBoard) and health metrics.

Behaviour parity with ``src/forgeline/observability/metrics.py:35-199``: the
local sink appends ``metrics.jsonl`` / ``events.jsonl`` in the run directory
and writes non-finite floats as ``null``.
"""

from __future__ import annotations

import json
import math
import time
from pathlib import Path
from typing import Any, Dict, List, Mapping, Optional

import torch

from rl_project_b200.core.errors import ConfigError, OptionalDependencyError


def _numeric(metrics: Mapping[str, Any]) -> Dict[str, float]:
    out: Dict[str, float] = {}
    for key, val in metrics.items():
        if isinstance(val, torch.Tensor):
            val = float(val.detach().float().mean().item())
        if isinstance(val, bool):
            val = float(val)
        if isinstance(val, (int, float)):
            out[key] = float(val)
    return out


def _json_safe(record: Mapping[str, Any]) -> Dict[str, Any]:
    return {k: (None if isinstance(v, float) and not math.isfinite(v) else v) for k, v in record.items()}


class MetricsSink:
    backend = "memory"

    def __init__(self) -> None:
        self.history: List[Dict[str, Any]] = []
        self.events: List[Dict[str, Any]] = []
        self.counters: Dict[str, int] = {}
        self._step = 0

    def log(self, metrics: Mapping[str, Any], step: Optional[int] = None) -> None:
        if step is not None:
            self._step = int(step)
        rec = {"step": self._step, "ts": time.time(), **_numeric(metrics)}
        self.history.append(rec)
        self._write(rec)

    def event(self, name: str, payload: Optional[Mapping[str, Any]] = None) -> None:
        rec = {"event": name, "ts": time.time(), "step": self._step, **dict(payload or {})}
        self.events.append(rec)
        self._write_event(rec)

    def increment(self, counter: str, by: int = 1) -> int:
        self.counters[counter] = self.counters.get(counter, 0) + by
        return self.counters[counter]

    def latest(self, key: str) -> Optional[float]:
        for rec in reversed(self.history):
            if key in rec:
                return rec[key]
        return None

    def series(self, key: str) -> List[float]:
        return [rec[key] for rec in self.history if key in rec]

    def _write(self, record: Mapping[str, Any]) -> None:
        pass

    def _write_event(self, record: Mapping[str, Any]) -> None:
        pass

    def close(self) -> None:
        pass


class NoOpMetricsSink(MetricsSink):
    backend = "noop"


class LocalJsonlMetricsSink(MetricsSink):
    backend = "local"

    def __init__(self, output_dir: str | Path, run_name: str = "run"):
        super().__init__()
        self.output_dir = Path(output_dir)
        self.output_dir.mkdir(parents=True, exist_ok=True)
        self.metrics_path = self.output_dir / "metrics.jsonl"
        self.events_path = self.output_dir / "events.jsonl"
        self.run_name = run_name

    def _append(self, path: Path, record: Mapping[str, Any]) -> None:
        with path.open("a") as fh:
            fh.write(json.dumps(_json_safe(record), default=str) + "\n")

    def _write(self, record: Mapping[str, Any]) -> None:
        self._append(self.metrics_path, record)

    def _write_event(self, record: Mapping[str, Any]) -> None:
        self._append(self.events_path, record)


class WandbMetricsSink(MetricsSink):
    backend = "wandb"

    def __init__(self, project: str, run_name: str, config: Optional[Mapping[str, Any]] = None):
        super().__init__()
        try:
            import wandb
        except ImportError as exc:
            raise OptionalDependencyError("wandb is not installed", hint="pip install wandb") from exc
        self._wandb = wandb
        self._run = wandb.init(project=project, name=run_name, config=dict(config or {}), resume="allow")

    def _write(self, record: Mapping[str, Any]) -> None:
        self._wandb.log({k: v for k, v in record.items() if k != "ts"}, step=int(record["step"]))

    def close(self) -> None:
        self._wandb.finish()


class TensorBoardMetricsSink(MetricsSink):
    backend = "tensorboard"

    def __init__(self, log_dir: str | Path):
        super().__init__()
        try:
            from torch.utils.tensorboard import SummaryWriter
        except ImportError as exc:
            raise OptionalDependencyError("tensorboard is not installed", hint="pip install tensorboard") from exc
        self._writer = SummaryWriter(log_dir=str(log_dir))

    def _write(self, record: Mapping[str, Any]) -> None:
        for key, val in record.items():
            if key not in ("step", "ts"):
                self._writer.add_scalar(key, val, int(record["step"]))

    def close(self) -> None:
        self._writer.close()


def build_metrics_sink(backend: str, *, output_dir: str | Path = "runs", run_name: str = "run",
                       project: str = "forgeline", config: Optional[Mapping[str, Any]] = None) -> MetricsSink:
    if backend in ("local", "jsonl"):
        return LocalJsonlMetricsSink(output_dir, run_name)
    if backend in ("none", "noop", "memory"):
        return NoOpMetricsSink()
    if backend == "wandb":
        return WandbMetricsSink(project, run_name, config)
    if backend == "tensorboard":
        return TensorBoardMetricsSink(Path(output_dir) / "tensorboard")
    raise ConfigError(f"Unknown metrics backend {backend!r}; use local|none|wandb|tensorboard")


def gradient_norms(model: torch.nn.Module, keys: tuple = ("wte", "ln_f", "lm_head")) -> Dict[str, float]:
    out: Dict[str, float] = {}
    sq = 0.0
    for name, p in model.named_parameters():
        if p.grad is None:
            continue
        n = float(p.grad.detach().float().norm(2).item())
        sq += n * n
        if any(k in name for k in keys):
            out[f"grad_norm/{name}"] = n
    out["grad_norm/total"] = math.sqrt(sq)
    return out


def device_memory_metrics(device: torch.device) -> Dict[str, float]:
    if device.type != "cuda":
        return {}
    return {
        "memory/allocated_gb": torch.cuda.memory_allocated(device) / 1e9,
        "memory/reserved_gb": torch.cuda.memory_reserved(device) / 1e9,
        "memory/max_allocated_gb": torch.cuda.max_memory_allocated(device) / 1e9,
    }


def perf_metrics(tokens: int, seconds: float, n_params: int, peak_tflops: float = 0.0,
                 world_size: int = 1) -> Dict[str, float]:
    """``perf/*`` metrics: tokens/s, model TFLOP/s (6N per token) and MFU against a peak."""
    if seconds <= 0:
        return {}
    tps = tokens / seconds
    tflops = 6.0 * n_params * tps / 1e12
    out = {"perf/tokens_per_s": tps, "perf/model_tflops": tflops}
    if peak_tflops > 0:
        out["perf/mfu"] = tflops / (peak_tflops * world_size)
    return out
