"""Rollouts: sampling engines (single-turn, agent/tool), verifiers, reward providers."""

from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine, stack_group, stack_old_logprobs
