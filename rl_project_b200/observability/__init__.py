"""Structured logging, metrics sinks, lifecycle events, timing spans and device timers."""

from rl_project_b200.observability.events import Event
from rl_project_b200.observability.logging import configure_logging, get_logger
from rl_project_b200.observability.metrics import (
    LocalJsonlMetricsSink,
    MetricsSink,
    NoOpMetricsSink,
    build_metrics_sink,
    device_memory_metrics,
    gradient_norms,
)
from rl_project_b200.observability.tracing import CudaTimer, Tracer, global_tracer, nvtx_range
