"""Reward providers: rules, verifier adapters, composites, process rewards, critics, learned models.

``build_reward_provider`` reads a manifest ``reward`` mapping
(``src/forgeline/rollouts/rewards/__init__.py:16-56`` keys)."""

from typing import Any, Dict

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.rollouts.rewards.composite import (CallableReward, CompositeReward, TagFormatReward,
                                                        VerifierReward, score_trajectories)
from rl_project_b200.rollouts.rewards.critic import CriticReward, heuristic_critic_score
from rl_project_b200.rollouts.rewards.learned import BlendedReward, RewardModelProvider
from rl_project_b200.rollouts.rewards.process import ProcessReward, compute_process_reward, parse_steps, score_step
from rl_project_b200.rollouts.rewards.rules import ConstantReward, LengthReward, RepetitionReward, TextFormatReward
from rl_project_b200.rollouts.verifiers import build_verifier

RULE_REWARDS = {"length": LengthReward, "text_format": TextFormatReward, "repetition": RepetitionReward,
                "constant": ConstantReward}


def build_reward_provider(config: Dict[str, Any]):
    kind = config.get("type")
    if kind == "verifier":
        params = {k: v for k, v in config.items() if k not in ("type", "verifier", "target_key", "weight")}
        return VerifierReward(build_verifier(config["verifier"], **params), target_key=config.get("target_key", "answer"),
                              weight=float(config.get("weight", 1.0)))
    if kind == "rule":
        return RULE_REWARDS[config["name"]](**{k: v for k, v in config.items() if k not in ("type", "name", "weight")})
    if kind == "composite":
        provs = [(build_reward_provider({k: v for k, v in p.items() if k != "weight"}), float(p.get("weight", 1.0)))
                 for p in config["providers"]]
        return CompositeReward(provs, clip=tuple(config["clip"]) if config.get("clip") else None)
    if kind == "process":
        return ProcessReward(float(config.get("gamma", 0.9)), float(config.get("step_weight", 1.0)),
                             config.get("target_key", "answer"), bool(config.get("execute_code", True)))
    if kind == "tagged":
        base = VerifierReward(build_verifier("tagged_answer"), target_key=config.get("target_key", "answer"))
        if config.get("format_bonus", True):
            return CompositeReward([(base, 1.0), (TagFormatReward(), 1.0)], name="tagged+format")
        return base
    if kind == "critic":
        return CriticReward(mode=config.get("mode", "heuristic"))
    if kind == "synthesis_rule":
        from rl_project_b200.domains.synthesis.reward import SynthesisRuleReward

        return SynthesisRuleReward(decode_from_text=bool(config.get("decode_from_text", True)))
    raise ConfigError(f"unknown reward type {kind!r}")
