"""Target-free rule rewards (``src/forgeline/rollouts/rewards/rules.py``)."""

from __future__ import annotations

from rl_project_b200.core.protocols import RewardResult, Trajectory


class LengthReward:
    name = "length"

    def __init__(self, target_length: int = 100):
        self.target_length = target_length

    def score(self, trajectory: Trajectory) -> RewardResult:
        gap = abs(trajectory.response_length - self.target_length)
        return RewardResult(max(0.0, 1.0 - gap / self.target_length))


class TextFormatReward:
    name = "text_format"

    def score(self, trajectory: Trajectory) -> RewardResult:
        t = trajectory.response_text
        return RewardResult(0.3 * ("." in t) + 0.3 * ("\n" in t) + 0.2 * (len(t) > 20) + 0.2 * bool(t.strip()))


class RepetitionReward:
    name = "repetition"

    def score(self, trajectory: Trajectory) -> RewardResult:
        toks = trajectory.response_ids.tolist()
        if len(toks) < 4:
            return RewardResult(0.5)
        pairs = list(zip(toks, toks[1:]))
        return RewardResult(len(set(pairs)) / max(len(pairs), 1))


class ConstantReward:
    name = "constant"

    def __init__(self, value: float = 0.0):
        self.value = value

    def score(self, trajectory: Trajectory) -> RewardResult:
        return RewardResult(self.value)
