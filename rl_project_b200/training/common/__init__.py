"""Shared training lifecycle and numerical utilities."""

from rl_project_b200.training.common.advantages import compute_gae, group_relative_advantages, normalize_advantages
from rl_project_b200.training.common.optim import build_optimizer
from rl_project_b200.training.common.precision import Precision
from rl_project_b200.training.common.schedule import learning_rate_at
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm, StepResult, Trainer
