"""RLVR: GRPO or DAPO driven by deterministic verifiers (``src/forgeline/training/rlvr.py``)."""

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
        if self.optimizer not in ("dapo", "grpo"):
            raise ConfigError("RLVR optimizer must be dapo|grpo")
        if self.task_type not in ("math", "code", "tagged_answer", "exact_match", "last_token_parity"):
            raise ConfigError("task_type must be math|code|tagged_answer|exact_match|last_token_parity")


def build_verifiable_reward(cfg: RLVRConfig):
    key = "test_code" if cfg.task_type == "code" else "answer"
    correct = VerifierReward(build_verifier(cfg.task_type, **cfg.verifier_params), target_key=key)
    if not cfg.require_format:
        return correct
    fmt = VerifierReward(FormatVerifier(cfg.format_spec), target_key="format_spec")
    return CompositeReward([(correct, cfg.correctness_weight), (fmt, cfg.format_weight)], name="rlvr")


def build_rlvr_algorithm(policy, tasks: Sequence, cfg: RLVRConfig, rollout: Optional[RolloutConfig] = None):
    cfg.validate()
    reward = build_verifiable_reward(cfg)
    task_dicts = [t.to_dict() for t in tasks]
    for d in task_dicts:
        d.setdefault("format_spec", cfg.format_spec)
    prompts = [torch.tensor(policy.encode(t.prompt), dtype=torch.long) for t in tasks]
    alg = (DAPOAlgorithm(policy, prompts, reward, cfg.dapo, rollout, tasks=task_dicts) if cfg.optimizer == "dapo"
           else GRPOAlgorithm(policy, prompts, reward, cfg.grpo, rollout, tasks=task_dicts))
    alg.name = "rlvr"
    return alg


@torch.no_grad()
def evaluate_pass_rate(policy, tasks: Sequence, reward, max_new_tokens: int = 64, temperature: float = 0.0,
                       limit: Optional[int] = None) -> Dict[str, float]:
    engine = RolloutEngine(policy, RolloutConfig(group_size=1, max_new_tokens=max_new_tokens, temperature=temperature,
                                                 record_old_logprobs=False))
    n = passed = malformed = 0
    total = 0.0
    for task in list(tasks)[: limit or None]:
        t = engine.rollout(torch.tensor(policy.encode(task.prompt)), task.to_dict())[0]
        r = reward.score(t)
        n += 1
        total += r.value
        passed += int(bool(r.passed))
        if r.info.get("predicted", "x") is None or "error" in r.info:
            malformed += 1
    return {"pass_rate": passed / max(n, 1), "reward": total / max(n, 1), "malformed_rate": malformed / max(n, 1),
            "n": n}
