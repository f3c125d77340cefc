"""Reward providers: rules, verifier adapters, composites, process rewards, critics and learned models.

``build_reward_provider`` turns a manifest ``reward`` mapping into a provider (the ``type`` values and keys
of ``src/forgeline/rollouts/rewards/__init__.py``) through the ``_BUILDERS`` table: ``verifier``, ``rule``,
``composite`` (members built recursively, each with its ``weight``), ``process``, ``tagged`` (tagged-answer
verifier plus the tag-format bonus unless ``format_bonus`` is false), ``critic`` and ``synthesis_rule``.
"""

from typing import Any, Callable, Dict

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.rollouts.rewards.composite import (CallableReward, CompositeReward, TagFormatReward,
                                                        VerifierReward, batch_scores, score_trajectories)
from rl_project_b200.rollouts.rewards.critic import CriticReward, heuristic_critic_score
from rl_project_b200.rollouts.rewards.learned import BlendedReward, RewardModelProvider
from rl_project_b200.rollouts.rewards.process import ProcessReward, compute_process_reward, parse_steps, score_step
from rl_project_b200.rollouts.rewards.rules import ConstantReward, LengthReward, RepetitionReward, TextFormatReward
from rl_project_b200.rollouts.verifiers import build_verifier

RULE_REWARDS = {"length": LengthReward, "text_format": TextFormatReward, "repetition": RepetitionReward,
                "constant": ConstantReward}


def _without(cfg: Dict[str, Any], *keys: str) -> Dict[str, Any]:
    return {k: v for k, v in cfg.items() if k not in keys}


def _verifier(cfg):
    params = _without(cfg, "type", "verifier", "target_key", "weight")
    return VerifierReward(build_verifier(cfg["verifier"], **params), target_key=cfg.get("target_key", "answer"),
                          weight=float(cfg.get("weight", 1.0)))


def _rule(cfg):
    return RULE_REWARDS[cfg["name"]](**_without(cfg, "type", "name", "weight"))


def _composite(cfg):
    members = [(build_reward_provider(_without(m, "weight")), float(m.get("weight", 1.0))) for m in cfg["providers"]]
    return CompositeReward(members, clip=tuple(cfg["clip"]) if cfg.get("clip") else None)


def _process(cfg):
    return ProcessReward(float(cfg.get("gamma", 0.9)), float(cfg.get("step_weight", 1.0)),
                         cfg.get("target_key", "answer"), bool(cfg.get("execute_code", True)))


def _tagged(cfg):
    answer = VerifierReward(build_verifier("tagged_answer"), target_key=cfg.get("target_key", "answer"))
    if not cfg.get("format_bonus", True):
        return answer
    return CompositeReward([(answer, 1.0), (TagFormatReward(), 1.0)], name="tagged+format")


def _synthesis(cfg):
    from rl_project_b200.domains.synthesis.reward import SynthesisRuleReward

    return SynthesisRuleReward(decode_from_text=bool(cfg.get("decode_from_text", True)))


_BUILDERS: Dict[str, Callable[[Dict[str, Any]], Any]] = {
    "verifier": _verifier, "rule": _rule, "composite": _composite, "process": _process, "tagged": _tagged,
    "critic": lambda cfg: CriticReward(mode=cfg.get("mode", "heuristic")), "synthesis_rule": _synthesis,
}


def build_reward_provider(config: Dict[str, Any]):
    build = _BUILDERS.get(config.get("type"))
    if build is None:
        raise ConfigError(f"unknown reward type {config.get('type')!r}")
    return build(config)
