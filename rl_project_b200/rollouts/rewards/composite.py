"""Reward composition (class names and the ``score_trajectories`` contract of
``src/forgeline/rollouts/rewards/composite.py``).

Providers here are batch-first: ``score_many(trajectories)`` is the primary entry and ``score`` is the
one-item case.  A ``CompositeReward`` asks each member for the whole batch at once -- so a verifier that
runs programs runs all of them concurrently, and a learned reward model does one forward -- and then
combines the per-trajectory values (weighted sum, optional clip; ``passed`` from the first member that
reports one).  ``score_trajectories`` rejects a non-finite value with ``InvalidRewardError`` and stores
each result on its trajectory.
"""

from __future__ import annotations

import math
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

from rl_project_b200.core.errors import InvalidRewardError
from rl_project_b200.core.protocols import RewardProvider, RewardResult, Trajectory, Verifier
from rl_project_b200.rollouts.verifiers import tag_format_reward


def _finite(value: Any, source: str) -> float:
    if not isinstance(value, (int, float)) or not math.isfinite(float(value)):
        raise InvalidRewardError(f"reward provider {source!r} returned non-finite value {value!r}")
    return float(value)


def batch_scores(provider: RewardProvider, trajectories: Sequence[Trajectory]) -> List[RewardResult]:
    """The provider's results for a batch (its ``score_many`` when it has one)."""
    many = getattr(provider, "score_many", None)
    return list(many(list(trajectories))) if callable(many) else [provider.score(t) for t in trajectories]


class _BatchFirst:
    name = "reward"

    def score_many(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        raise NotImplementedError

    def score(self, trajectory: Trajectory) -> RewardResult:
        return self.score_many([trajectory])[0]


class VerifierReward(_BatchFirst):
    """A verifier applied to the response text (or its token ids, for token-level rules) against
    ``task[target_key]``, scaled by ``weight``."""

    def __init__(self, verifier: Verifier, target_key: str = "answer", weight: float = 1.0, on_tokens: bool = False):
        self.verifier, self.target_key, self.weight = verifier, target_key, weight
        self.on_tokens = on_tokens or getattr(verifier, "name", "") == "last_token_parity"
        self.name = f"verifier:{verifier.name}"

    def score_many(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        outputs = [t.response_ids if self.on_tokens else t.response_text for t in trajectories]
        targets = [t.task.get(self.target_key) for t in trajectories]
        many = getattr(self.verifier, "verify_many", None)
        raw = many(outputs, targets) if callable(many) else [self.verifier.verify(o, g) for o, g in zip(outputs, targets)]
        return [RewardResult(_finite(r.value, self.name) * self.weight, passed=r.passed,
                             components={self.name: r.value}, info=r.info) for r in raw]


class TagFormatReward(_BatchFirst):
    name = "tag_format"

    def score_many(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        return [RewardResult(tag_format_reward(t.response_text)) for t in trajectories]


class CompositeReward(_BatchFirst):
    def __init__(self, providers: Sequence[Tuple[RewardProvider, float]], name: str = "composite",
                 clip: Optional[Tuple[float, float]] = None):
        if not providers:
            raise InvalidRewardError("composite reward needs at least one provider")
        self.providers, self.name, self.clip = list(providers), name, clip

    def score_many(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        columns = [(prov, w, batch_scores(prov, trajectories)) for prov, w in self.providers]
        out = []
        for i in range(len(trajectories)):
            comps: Dict[str, float] = {}
            info: Dict[str, Any] = {}
            total, passed = 0.0, None
            for prov, w, results in columns:
                r = results[i]
                v = _finite(r.value, prov.name)
                comps[prov.name] = v
                total += w * v
                passed = r.passed if passed is None else passed
                if r.info:
                    info[prov.name] = r.info
            if self.clip is not None:
                total = min(max(total, self.clip[0]), self.clip[1])
            out.append(RewardResult(total, components=comps, passed=passed, info=info))
        return out


class CallableReward(_BatchFirst):
    def __init__(self, fn: Callable[[Trajectory], float], name: str = "callable"):
        self.fn, self.name = fn, name

    def score_many(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        return [RewardResult(_finite(self.fn(t), self.name)) for t in trajectories]


def score_trajectories(provider: RewardProvider, trajectories: List[Trajectory]) -> List[float]:
    values = []
    for t, r in zip(trajectories, batch_scores(provider, trajectories)):
        _finite(r.value, provider.name)
        t.reward = r
        values.append(r.value)
    return values
