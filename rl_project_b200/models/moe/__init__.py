"""Mixture-of-experts routing and layers."""

from rl_project_b200.models.moe.gate import ExpertGate
from rl_project_b200.models.moe.layer import MoELayer, sort_by_expert
