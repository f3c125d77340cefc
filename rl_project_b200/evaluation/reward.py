"""Reward evaluation suites (suite names, metric keys and the ``policy_dependent`` flag of
``src/forgeline/evaluation/reward.py``): reward statistics over dataset records (a property of the data)
or policy trajectories, and the preference win rate of a scorer.

Statistics are computed on one float64 array: mean, population std, min, max, the improvement over a
baseline in percent, and the percentage above each threshold.
"""

from __future__ import annotations

from typing import Any, Callable, Dict, Sequence

import numpy as np

from rl_project_b200.core.protocols import EvaluationResult, RewardProvider, Trajectory


def reward_statistics(rewards: Sequence[float], baseline: float = 0.5,
                      thresholds: Sequence[float] = (0.6, 0.75)) -> Dict[str, float]:
    r = np.asarray(list(rewards), dtype=np.float64)
    if r.size == 0:
        return {"mean": 0.0, "std": 0.0, "min": 0.0, "max": 0.0, "n": 0}
    mean = float(r.mean())
    stats = {"mean": mean, "std": float(r.std()), "min": float(r.min()), "max": float(r.max()), "n": float(r.size),
             "improvement_vs_baseline_pct": 100.0 * (mean - baseline) / baseline if baseline else 0.0}
    stats.update({f"pct_above_{t}": 100.0 * float((r > t).mean()) for t in thresholds})
    return stats


def _result(name: str, rewards: Sequence[float], baseline: float, policy_dependent: bool) -> EvaluationResult:
    return EvaluationResult(name, reward_statistics(rewards, baseline), n_samples=len(rewards),
                            details={"policy_dependent": policy_dependent})


class RecordRewardSuite:
    """Scores dataset records: measures the data, not a policy."""

    name = "record_reward"

    def __init__(self, records: Sequence[Dict[str, Any]], score_fn: Callable[[Dict[str, Any]], float],
                 baseline: float = 0.5):
        self.records, self.score_fn, self.baseline = list(records), score_fn, baseline

    def run(self, target: Any = None, **kwargs: Any) -> EvaluationResult:
        return _result(self.name, [float(self.score_fn(r)) for r in self.records], self.baseline, False)


class TrajectoryRewardSuite:
    name = "trajectory_reward"

    def __init__(self, reward: RewardProvider, baseline: float = 0.5):
        self.reward, self.baseline = reward, baseline

    def run(self, trajectories: Sequence[Trajectory], **kwargs: Any) -> EvaluationResult:
        from rl_project_b200.rollouts.rewards.composite import batch_scores

        values = [float(r.value) for r in batch_scores(self.reward, list(trajectories))]
        return _result(self.name, values, self.baseline, True)


class PreferenceWinRateSuite:
    """Fraction of pairs whose ``chosen`` side the scorer ranks above ``rejected``, and the mean margin."""

    name = "preference_win_rate"

    def __init__(self, pairs: Sequence[Dict[str, str]], score_fn: Callable[[str, str], float]):
        self.pairs, self.score_fn = list(pairs), score_fn

    def run(self, target: Any = None, **kwargs: Any) -> EvaluationResult:
        margin = np.asarray([float(self.score_fn(p["prompt"], p["chosen"])) - float(self.score_fn(p["prompt"], p["rejected"]))
                             for p in self.pairs], dtype=np.float64)
        n = max(len(self.pairs), 1)
        return EvaluationResult(self.name, {"win_rate": float((margin > 0).sum()) / n,
                                            "mean_margin": float(margin.sum()) / n}, n_samples=len(self.pairs))
