"""Rewards from learned models (``src/forgeline/rollouts/rewards/learned.py``)."""

from __future__ import annotations

from typing import Callable, List, Optional

import torch

from rl_project_b200.core.protocols import RewardResult, Trajectory


class RewardModelProvider:
    name = "reward_model"

    def __init__(self, model, max_length: Optional[int] = None):
        self.model = model.eval()
        self.max_length = max_length or model.spec.block_size

    @torch.no_grad()
    def score(self, trajectory: Trajectory) -> RewardResult:
        return self.score_many([trajectory])[0]

    @torch.no_grad()
    def score_many(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        dev = next(self.model.parameters()).device
        out = []
        for t in trajectories:
            ids = torch.cat([t.prompt_ids, t.response_ids])[None, -self.max_length:].to(dev)
            out.append(RewardResult(float(self.model(ids).float().item())))
        return out


class BlendedReward:
    name = "blended"

    def __init__(self, rule_fn: Callable[[Trajectory], float], neural: Optional[Callable[[Trajectory], float]] = None,
                 neural_weight: float = 0.6):
        self.rule_fn, self.neural, self.neural_weight = rule_fn, neural, neural_weight

    def score(self, trajectory: Trajectory) -> RewardResult:
        rule = float(self.rule_fn(trajectory))
        if self.neural is None:
            return RewardResult(rule, components={"rule": rule})
        neural = float(self.neural(trajectory))
        v = max(0.0, min(1.0, (1 - self.neural_weight) * rule + self.neural_weight * neural))
        return RewardResult(v, components={"rule": rule, "neural": neural})
