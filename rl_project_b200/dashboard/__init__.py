"""Local read-only dashboard: runs, checkpoints, evaluations, registry, benchmarks, model inspection."""

from rl_project_b200.dashboard.data import DashboardSources, snapshot
from rl_project_b200.dashboard.server import DashboardApp, DashboardServer

__all__ = ["DashboardSources", "snapshot", "DashboardApp", "DashboardServer"]
