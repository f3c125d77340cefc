"""Rewards from learned models (the providers of ``src/forgeline/rollouts/rewards/learned.py``).

``RewardModelProvider`` scores a whole batch with one forward of the sequence reward model: each
trajectory's ``prompt + response`` ids (the last ``max_length`` of them) are right-padded into one
``[B, T]`` tensor and the attention mask tells the model's pooling where each row ends.
``BlendedReward`` mixes a rule score with a neural score and clips to [0, 1].
"""

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
    def score_many(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        if not trajectories:
            return []
        dev = next(self.model.parameters()).device
        rows = [torch.cat([t.prompt_ids, t.response_ids])[-self.max_length:] for t in trajectories]
        width = max(r.numel() for r in rows)
        ids = torch.zeros(len(rows), width, dtype=torch.long)
        mask = torch.zeros(len(rows), width, dtype=torch.long)
        for i, r in enumerate(rows):
            ids[i, :r.numel()] = r
            mask[i, :r.numel()] = 1
        scores = self.model(ids.to(dev), mask.to(dev)).float().cpu().tolist()
        return [RewardResult(v) for v in scores]

    def score(self, trajectory: Trajectory) -> RewardResult:
        return self.score_many([trajectory])[0]


class BlendedReward:
    name = "blended"

    def __init__(self, rule_fn: Callable[[Trajectory], float], neural: Optional[Callable[[Trajectory], float]] = None,
                 neural_weight: float = 0.6):
        self.rule_fn, self.neural, self.neural_weight = rule_fn, neural, neural_weight

    def score(self, trajectory: Trajectory) -> RewardResult:
        rule = float(self.rule_fn(trajectory))
        parts = {"rule": rule}
        if self.neural is None:
            return RewardResult(rule, components=parts)
        parts["neural"] = float(self.neural(trajectory))
        mixed = (1.0 - self.neural_weight) * parts["rule"] + self.neural_weight * parts["neural"]
        return RewardResult(min(1.0, max(0.0, mixed)), components=parts)
