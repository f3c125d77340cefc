"""RLVR: policy optimisation against deterministic verifiers (the capability of
``src/forgeline/training/rlvr.py``).

An RLVR run is GRPO or DAPO whose reward is a verifier's pass/fail score on each task's target
(``answer``, or ``test_code`` for code tasks), optionally blended with a format check.  The pieces are
looked up in two tables below rather than branched on; ``evaluate_pass_rate`` answers every evaluation
task in one batched rollout call and scores the whole batch.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, Optional, Sequence

import torch

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine
from rl_project_b200.rollouts.rewards.composite import CompositeReward, VerifierReward
from rl_project_b200.rollouts.verifiers import FormatVerifier, build_verifier
from rl_project_b200.training.dapo import DAPOAlgorithm, DAPOConfig
from rl_project_b200.training.grpo import GRPOAlgorithm, GRPOConfig

# task type -> the task field its verifier checks the response against
TARGET_FIELD: Dict[str, str] = {"math": "answer", "code": "test_code", "tagged_answer": "answer",
                                "exact_match": "answer", "last_token_parity": "answer"}


@dataclass
class RLVRConfig:
    task_type: str = "math"
    optimizer: str = "dapo"
    require_format: bool = False
    format_spec: str = "cot"
    correctness_weight: float = 0.7
    format_weight: float = 0.3
    verifier_params: Dict[str, Any] = field(default_factory=dict)
    grpo: GRPOConfig = field(default_factory=GRPOConfig)
    dapo: DAPOConfig = field(default_factory=DAPOConfig)

    def validate(self) -> None:
        if self.optimizer not in _ALGORITHMS:
            raise ConfigError(f"RLVR optimizer must be {'|'.join(_ALGORITHMS)}")
        if self.task_type not in TARGET_FIELD:
            raise ConfigError(f"task_type must be {'|'.join(TARGET_FIELD)}")


def build_verifiable_reward(cfg: RLVRConfig):
    """The verifier's score on the task target, or its weighted blend with the format check."""
    correctness = VerifierReward(build_verifier(cfg.task_type, **cfg.verifier_params),
                                 target_key=TARGET_FIELD[cfg.task_type])
    if not cfg.require_format:
        return correctness
    layout = VerifierReward(FormatVerifier(cfg.format_spec), target_key="format_spec")
    return CompositeReward([(correctness, cfg.correctness_weight), (layout, cfg.format_weight)], name="rlvr")


# optimizer name -> (algorithm class, the RLVRConfig field holding its config)
_ALGORITHMS = {"dapo": (DAPOAlgorithm, "dapo"), "grpo": (GRPOAlgorithm, "grpo")}


def build_rlvr_algorithm(policy, tasks: Sequence, cfg: RLVRConfig, rollout: Optional[RolloutConfig] = None):
    cfg.validate()
    records = [{"format_spec": cfg.format_spec, **t.to_dict()} for t in tasks]
    prompts = [torch.tensor(policy.encode(t.prompt), dtype=torch.long) for t in tasks]
    cls, sub = _ALGORITHMS[cfg.optimizer]
    algorithm = cls(policy, prompts, build_verifiable_reward(cfg), getattr(cfg, sub), rollout, tasks=records)
    algorithm.name = "rlvr"
    return algorithm


@torch.no_grad()
def evaluate_pass_rate(policy, tasks: Sequence, reward, max_new_tokens: int = 64, temperature: float = 0.0,
                       limit: Optional[int] = None) -> Dict[str, float]:
    """Pass rate, mean reward and malformed-answer rate of one sampled answer per task (all tasks in one batched
    rollout).  An answer is malformed when the verifier could not extract a prediction or raised."""
    chosen = list(tasks)[: limit or None]
    if not chosen:
        return {"pass_rate": 0.0, "reward": 0.0, "malformed_rate": 0.0, "n": 0}
    engine = RolloutEngine(policy, RolloutConfig(group_size=1, max_new_tokens=max_new_tokens, temperature=temperature,
                                                 record_old_logprobs=False))
    groups = engine.rollout_many([torch.tensor(policy.encode(t.prompt), dtype=torch.long) for t in chosen],
                                 [t.to_dict() for t in chosen])
    scores = [reward.score(grp[0]) for grp in groups]
    n = len(scores)
    malformed = sum(1 for s in scores if s.info.get("predicted", "x") is None or "error" in s.info)
    return {"pass_rate": sum(bool(s.passed) for s in scores) / n, "reward": sum(s.value for s in scores) / n,
            "malformed_rate": malformed / n, "n": n}
