"""Reward statistics over dataset records, policy trajectories and preference pairs
(``src/forgeline/evaluation/reward.py:11-72`` metrics and keys)."""

from __future__ import annotations

import math
from typing import Any, Callable, Dict, List, Sequence

from rl_project_b200.core.protocols import EvaluationResult, RewardProvider, Trajectory


def reward_statistics(rewards: Sequence[float], baseline: float = 0.5,
                      thresholds: Sequence[float] = (0.6, 0.75)) -> Dict[str, float]:
    if not rewards:
        return {"mean": 0.0, "std": 0.0, "min": 0.0, "max": 0.0, "n": 0}
    n = len(rewards)
    mean = math.fsum(rewards) / n
    out = {"mean": mean, "std": math.sqrt(math.fsum((r - mean) ** 2 for r in rewards) / n),
           "min": min(rewards), "max": max(rewards), "n": float(n),
           "improvement_vs_baseline_pct": (mean - baseline) / baseline * 100.0 if baseline else 0.0}
    for t in thresholds:
        out[f"pct_above_{t}"] = 100.0 * sum(r > t for r in rewards) / n
    return out


class RecordRewardSuite:
    """Scores dataset records with a scorer: measures the data, not a policy (``policy_dependent`` False)."""

    name = "record_reward"

    def __init__(self, records: Sequence[Dict[str, Any]], score_fn: Callable[[Dict[str, Any]], float],
                 baseline: float = 0.5):
        self.records, self.score_fn, self.baseline = list(records), score_fn, baseline

    def run(self, target: Any = None, **kwargs: Any) -> EvaluationResult:
        rewards = [float(self.score_fn(r)) for r in self.records]
        return EvaluationResult(self.name, reward_statistics(rewards, self.baseline), n_samples=len(rewards),
                                details={"policy_dependent": False})


class TrajectoryRewardSuite:
    name = "trajectory_reward"

    def __init__(self, reward: RewardProvider, baseline: float = 0.5):
        self.reward, self.baseline = reward, baseline

    def run(self, trajectories: Sequence[Trajectory], **kwargs: Any) -> EvaluationResult:
        score_many = getattr(self.reward, "score_many", None)
        results = score_many(list(trajectories)) if score_many else [self.reward.score(t) for t in trajectories]
        rewards = [float(r.value) for r in results]
        return EvaluationResult(self.name, reward_statistics(rewards, self.baseline), n_samples=len(rewards),
                                details={"policy_dependent": True})


class PreferenceWinRateSuite:
    """Fraction of pairs whose ``chosen`` scores above ``rejected``, and the mean margin."""

    name = "preference_win_rate"

    def __init__(self, pairs: Sequence[Dict[str, str]], score_fn: Callable[[str, str], float]):
        self.pairs, self.score_fn = list(pairs), score_fn

    def run(self, target: Any = None, **kwargs: Any) -> EvaluationResult:
        margins: List[float] = [float(self.score_fn(p["prompt"], p["chosen"]) - self.score_fn(p["prompt"], p["rejected"]))
                                for p in self.pairs]
        n = max(len(self.pairs), 1)
        return EvaluationResult(self.name, {"win_rate": sum(m > 0 for m in margins) / n,
                                            "mean_margin": math.fsum(margins) / n}, n_samples=len(self.pairs))
