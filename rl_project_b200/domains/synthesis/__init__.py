"""Pharmaceutical-synthesis domain: record schema helpers, rule reward, constraints,
prompt / condition codec, state features, a seeded response-surface simulator,
preference / SFT record builders and a tabular actor-critic PPO baseline."""

from rl_project_b200.domains.synthesis.constraints import (CONDITION_BOUNDS, CONDITION_DEFAULTS, batch_validate,
                                                           validate_conditions, validity_penalty)
from rl_project_b200.domains.synthesis.features import encode_trajectory, molecule_fingerprint
from rl_project_b200.domains.synthesis.generator import predict_outcomes, simulate_dataset, yield_series_trajectories
from rl_project_b200.domains.synthesis.preferences import (build_preference_pairs, build_sft_records,
                                                           filter_high_reward, pairs_to_records)
from rl_project_b200.domains.synthesis.prompts import (CONDITION_KEYS, build_synthesis_prompt, conditions_to_json,
                                                       decode_conditions)
from rl_project_b200.domains.synthesis.reward import (RULE_WEIGHTS, SynthesisRuleReward, extract_outcomes,
                                                      rule_score, trajectory_to_text)
from rl_project_b200.domains.synthesis.tabular_ppo import (TabularActorCritic, TabularPPOConfig, TabularPPOTrainer,
                                                           load_trajectories)

__all__ = ["CONDITION_BOUNDS", "CONDITION_DEFAULTS", "batch_validate", "validate_conditions", "validity_penalty",
           "encode_trajectory", "molecule_fingerprint", "predict_outcomes", "simulate_dataset",
           "yield_series_trajectories", "build_preference_pairs", "build_sft_records", "filter_high_reward",
           "pairs_to_records", "CONDITION_KEYS", "build_synthesis_prompt", "conditions_to_json", "decode_conditions",
           "RULE_WEIGHTS", "SynthesisRuleReward", "extract_outcomes", "rule_score", "trajectory_to_text",
           "TabularActorCritic", "TabularPPOConfig", "TabularPPOTrainer", "load_trajectories"]
