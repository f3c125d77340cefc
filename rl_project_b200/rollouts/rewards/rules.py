"""Target-free rule rewards (the rules of ``src/forgeline/rollouts/rewards/rules.py``): closeness to a
target length, text-structure points, distinct-bigram ratio, a constant.

The bigram ratio works on the token tensor directly: consecutive pairs are packed into one int64 key
(``a * V + b`` with ``V`` above every id) and counted with ``torch.unique``.
"""

from __future__ import annotations

import torch

from rl_project_b200.core.protocols import RewardResult, Trajectory


class LengthReward:
    name = "length"

    def __init__(self, target_length: int = 100):
        self.target_length = target_length

    def score(self, trajectory: Trajectory) -> RewardResult:
        miss = abs(trajectory.response_length - self.target_length) / self.target_length
        return RewardResult(max(0.0, 1.0 - miss))


# (test on the decoded text, points)
_TEXT_POINTS = ((lambda t: "." in t, 0.3), (lambda t: "\n" in t, 0.3), (lambda t: len(t) > 20, 0.2),
                (lambda t: bool(t.strip()), 0.2))


class TextFormatReward:
    name = "text_format"

    def score(self, trajectory: Trajectory) -> RewardResult:
        text = trajectory.response_text
        return RewardResult(sum(points for test, points in _TEXT_POINTS if test(text)))


def distinct_bigram_ratio(tokens: torch.Tensor) -> float:
    t = tokens.reshape(-1).long()
    if t.numel() < 2:
        return 1.0
    base = int(t.max()) + 1
    keys = t[:-1] * base + t[1:]
    return torch.unique(keys).numel() / keys.numel()


class RepetitionReward:
    """Distinct-bigram ratio of the response tokens (0.5 for responses under four tokens)."""

    name = "repetition"

    def score(self, trajectory: Trajectory) -> RewardResult:
        ids = trajectory.response_ids
        return RewardResult(0.5 if ids.numel() < 4 else distinct_bigram_ratio(ids))


class ConstantReward:
    name = "constant"

    def __init__(self, value: float = 0.0):
        self.value = value

    def score(self, trajectory: Trajectory) -> RewardResult:
        return RewardResult(self.value)
