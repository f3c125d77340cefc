"""Parallelism: process groups, strategies (DDP / FSDP / ZeRO-2 / TP / PP / EP / 3-D mesh),
NVLink peer-memory communication kernels and the fused collective paths."""

from rl_project_b200.parallel.strategies import STRATEGIES, build_strategy
