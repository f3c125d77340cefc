"""Timing: host spans (``Tracer``), CUDA-event device timers and NVTX ranges.

``Tracer`` keeps the reference's span API (``src/forgeline/observability/tracing.py:11-57``).
``nvtx_range`` / ``nvtx_annotate`` name the fused communication paths and the
phases of a training step for a profiler (``RLB_NVTX=1``).
``CudaTimer`` measures on the device with CUDA events; ``max_over_ranks``
reduces a per-rank device time to the slowest rank, which is how every
multi-GPU number in this framework is reported.
"""

from __future__ import annotations

import functools
import os
import time
from collections import deque
from contextlib import contextmanager
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterator, List, Optional

import torch


@dataclass
class Span:
    name: str
    start: float
    end: Optional[float] = None
    attributes: Dict[str, object] = field(default_factory=dict)

    @property
    def duration_ms(self) -> float:
        stop = self.end if self.end is not None else time.time()
        return (stop - self.start) * 1e3


class Tracer:
    """Named spans.  The most recent ``keep`` spans are kept for inspection; the per-name
    aggregates (count / total / max) cover every span ever recorded, so a long-running
    server's memory stays bounded."""

    def __init__(self, keep: int = 10_000) -> None:
        self.spans: "deque[Span]" = deque(maxlen=keep)
        self._agg: Dict[str, Dict[str, float]] = {}

    @contextmanager
    def span(self, name: str, **attributes: object) -> Iterator[Span]:
        s = Span(name, time.time(), attributes=dict(attributes))
        try:
            yield s
        finally:
            s.end = time.time()
            self.spans.append(s)
            row = self._agg.setdefault(name, {"count": 0.0, "total_ms": 0.0, "max_ms": 0.0})
            d = s.duration_ms
            row["count"] += 1
            row["total_ms"] += d
            row["max_ms"] = max(row["max_ms"], d)

    def durations(self, name: str) -> List[float]:
        return [s.duration_ms for s in self.spans if s.name == name and s.end is not None]

    def summary(self) -> Dict[str, Dict[str, float]]:
        out = {k: dict(v) for k, v in self._agg.items()}
        for row in out.values():
            row["mean_ms"] = row["total_ms"] / max(1.0, row["count"])
        return out


_TRACER = Tracer()


def global_tracer() -> Tracer:
    return _TRACER


# NVTX ranges cost a host call each, so they are off unless RLB_NVTX=1 (or set_nvtx(True)): a profiler
# that reads NVTX then sees every fused communication path and the phases of a training step by name.
_NVTX = os.environ.get("RLB_NVTX", "0") == "1"


def set_nvtx(enabled: bool) -> None:
    global _NVTX
    _NVTX = bool(enabled)


def nvtx_enabled() -> bool:
    return _NVTX and torch.cuda.is_available()


@contextmanager
def nvtx_range(name: str) -> Iterator[None]:
    """A named NVTX range around the block (no-op unless NVTX ranges are enabled)."""
    if nvtx_enabled():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


def nvtx_annotate(name: str) -> Callable:
    """Decorator form of ``nvtx_range`` (the enable switch is read at call time)."""

    def wrap(fn: Callable) -> Callable:
        @functools.wraps(fn)
        def inner(*a, **k):
            if not _NVTX:
                return fn(*a, **k)
            with nvtx_range(name):
                return fn(*a, **k)

        return inner

    return wrap


class CudaTimer:
    """Device time between ``start()`` and ``stop()`` on the current stream (ms)."""

    def __init__(self) -> None:
        self._a = torch.cuda.Event(enable_timing=True)
        self._b = torch.cuda.Event(enable_timing=True)

    def start(self) -> None:
        self._a.record()

    def stop(self) -> float:
        self._b.record()
        self._b.synchronize()
        return float(self._a.elapsed_time(self._b))


def max_over_ranks(value: float, device: Optional[torch.device] = None) -> float:
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    dev = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
    if dist.get_backend() == "gloo":
        dev = torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
