"""Metrics sinks and training-health metrics (the sink classes, backends and file formats of
``src/forgeline/observability/metrics.py``: ``metrics.jsonl`` / ``events.jsonl`` in the run directory,
non-finite floats written as ``null``).

A sink is an in-memory history plus one *writer* (the destination: nothing, JSONL files, W&B or
TensorBoard); the public sink classes are the memory sink bound to their writer.  Device scalars in a
metrics dict are gathered and copied to the host in one transfer per ``log`` call (one synchronisation,
not one per tensor), and ``gradient_norms`` computes every parameter's norm with one fused multi-tensor
kernel and one transfer.
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
    """Plain floats: Python numbers and bools as they are, tensors as their mean (all fetched at once)."""
    out: Dict[str, float] = {}
    tensors: List[tuple] = []
    for key, val in metrics.items():
        if isinstance(val, torch.Tensor):
            tensors.append((key, val.detach().float().mean()))
        elif isinstance(val, (bool, int, float)):
            out[key] = float(val)
    if tensors:
        host = torch.stack([t.to(tensors[0][1].device) for _, t in tensors]).cpu().tolist()
        out.update({k: v for (k, _), v in zip(tensors, host)})
    return {k: out[k] for k in metrics if k in out}  # caller's key order


def _json_safe(record: Mapping[str, Any]) -> Dict[str, Any]:
    return {k: (None if isinstance(v, float) and not math.isfinite(v) else v) for k, v in record.items()}


class _Writer:
    """Destination of records; the base writes nowhere."""

    def metrics(self, record: Mapping[str, Any]) -> None:
        pass

    def event(self, record: Mapping[str, Any]) -> None:
        pass

    def close(self) -> None:
        pass


class _JsonlWriter(_Writer):
    def __init__(self, directory: Path):
        directory.mkdir(parents=True, exist_ok=True)
        self.paths = {"metrics": directory / "metrics.jsonl", "events": directory / "events.jsonl"}

    def _append(self, which: str, record: Mapping[str, Any]) -> None:
        with self.paths[which].open("a") as fh:
            fh.write(json.dumps(_json_safe(record), default=str) + "\n")

    def metrics(self, record):
        self._append("metrics", record)

    def event(self, record):
        self._append("events", record)


class _WandbWriter(_Writer):
    def __init__(self, project: str, run_name: str, config: Optional[Mapping[str, Any]]):
        try:
            import wandb
        except ImportError as exc:
            raise OptionalDependencyError("wandb is not installed", hint="pip install wandb") from exc
        self.wandb = wandb
        wandb.init(project=project, name=run_name, config=dict(config or {}), resume="allow")

    def metrics(self, record):
        self.wandb.log({k: v for k, v in record.items() if k != "ts"}, step=int(record["step"]))

    def close(self):
        self.wandb.finish()


class _TensorBoardWriter(_Writer):
    def __init__(self, log_dir: Path):
        try:
            from torch.utils.tensorboard import SummaryWriter
        except ImportError as exc:
            raise OptionalDependencyError("tensorboard is not installed", hint="pip install tensorboard") from exc
        self.tb = SummaryWriter(log_dir=str(log_dir))

    def metrics(self, record):
        step = int(record["step"])
        for k, v in record.items():
            if k not in ("step", "ts"):
                self.tb.add_scalar(k, v, step)

    def close(self):
        self.tb.close()


class MetricsSink:
    """History of metric records and events, counters, and the writer they go to."""

    backend = "memory"

    def __init__(self, writer: Optional[_Writer] = None) -> None:
        self.writer = writer or _Writer()
        self.history: List[Dict[str, Any]] = []
        self.events: List[Dict[str, Any]] = []
        self.counters: Dict[str, int] = {}
        self._step = 0

    def log(self, metrics: Mapping[str, Any], step: Optional[int] = None) -> None:
        if step is not None:
            self._step = int(step)
        record = {"step": self._step, "ts": time.time(), **_numeric(metrics)}
        self.history.append(record)
        self.writer.metrics(record)

    def event(self, name: str, payload: Optional[Mapping[str, Any]] = None) -> None:
        record = {"event": name, "ts": time.time(), "step": self._step, **dict(payload or {})}
        self.events.append(record)
        self.writer.event(record)

    def increment(self, counter: str, by: int = 1) -> int:
        self.counters[counter] = self.counters.get(counter, 0) + by
        return self.counters[counter]

    def series(self, key: str) -> List[float]:
        return [r[key] for r in self.history if key in r]

    def latest(self, key: str) -> Optional[float]:
        values = self.series(key)
        return values[-1] if values else None

    def close(self) -> None:
        self.writer.close()


class NoOpMetricsSink(MetricsSink):
    backend = "noop"


class LocalJsonlMetricsSink(MetricsSink):
    backend = "local"

    def __init__(self, output_dir: str | Path, run_name: str = "run"):
        self.output_dir, self.run_name = Path(output_dir), run_name
        super().__init__(_JsonlWriter(self.output_dir))
        self.metrics_path, self.events_path = self.writer.paths["metrics"], self.writer.paths["events"]


class WandbMetricsSink(MetricsSink):
    backend = "wandb"

    def __init__(self, project: str, run_name: str, config: Optional[Mapping[str, Any]] = None):
        super().__init__(_WandbWriter(project, run_name, config))


class TensorBoardMetricsSink(MetricsSink):
    backend = "tensorboard"

    def __init__(self, log_dir: str | Path):
        super().__init__(_TensorBoardWriter(Path(log_dir)))


_BACKENDS = {
    "local": lambda o: LocalJsonlMetricsSink(o["output_dir"], o["run_name"]),
    "jsonl": lambda o: LocalJsonlMetricsSink(o["output_dir"], o["run_name"]),
    "none": lambda o: NoOpMetricsSink(),
    "noop": lambda o: NoOpMetricsSink(),
    "memory": lambda o: NoOpMetricsSink(),
    "wandb": lambda o: WandbMetricsSink(o["project"], o["run_name"], o["config"]),
    "tensorboard": lambda o: TensorBoardMetricsSink(Path(o["output_dir"]) / "tensorboard"),
}


def build_metrics_sink(backend: str, *, output_dir: str | Path = "runs", run_name: str = "run",
                       project: str = "forgeline", config: Optional[Mapping[str, Any]] = None) -> MetricsSink:
    make = _BACKENDS.get(backend)
    if make is None:
        raise ConfigError(f"Unknown metrics backend {backend!r}; use local|none|wandb|tensorboard")
    return make({"output_dir": output_dir, "run_name": run_name, "project": project, "config": config})


def gradient_norms(model: torch.nn.Module, keys: tuple = ("wte", "ln_f", "lm_head")) -> Dict[str, float]:
    """``grad_norm/total`` over every gradient plus ``grad_norm/<name>`` for parameters whose name contains
    one of ``keys`` (norms of all gradients in one fused pass, one host transfer)."""
    named = [(n, p.grad) for n, p in model.named_parameters() if p.grad is not None]
    if not named:
        return {"grad_norm/total": 0.0}
    norms = torch._foreach_norm([g.detach().float() for _, g in named], 2)
    host = torch.stack([n.to(norms[0].device) for n in norms]).cpu()
    out = {f"grad_norm/{name}": float(v) for (name, _), v in zip(named, host.tolist()) if any(k in name for k in keys)}
    out["grad_norm/total"] = float(host.double().square().sum().sqrt())
    return out


def device_memory_metrics(device: torch.device) -> Dict[str, float]:
    if device.type != "cuda":
        return {}
    gb = 1e9
    return {"memory/allocated_gb": torch.cuda.memory_allocated(device) / gb,
            "memory/reserved_gb": torch.cuda.memory_reserved(device) / gb,
            "memory/max_allocated_gb": torch.cuda.max_memory_allocated(device) / gb}


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
