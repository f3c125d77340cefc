"""Budgeted sequential allocation: a POMDP simulator with latent policy-dependent
pressure, heuristic / dual-pacing / PPO (MLP, GRU) policies, logged episodes,
off-policy evaluation, hindsight oracle, simulated A/B and shadow experiments,
and an end-to-end benchmark."""

from rl_project_b200.domains.allocation.env import (ACTION_NAMES, MULTIPLIERS, OBS_DIM, AllocationEnvConfig,
                                                    BudgetedAllocationEnv, VectorEnv)
from rl_project_b200.domains.allocation.policies import (DualPacingPolicy, EpsilonMixPolicy, GRUActorCritic,
                                                         MLPActorCritic, NeuralPolicy, PolicyNetConfig,
                                                         ThresholdPacingPolicy)

__all__ = ["ACTION_NAMES", "MULTIPLIERS", "OBS_DIM", "AllocationEnvConfig", "BudgetedAllocationEnv", "VectorEnv",
           "DualPacingPolicy", "EpsilonMixPolicy", "GRUActorCritic", "MLPActorCritic", "NeuralPolicy",
           "PolicyNetConfig", "ThresholdPacingPolicy"]
