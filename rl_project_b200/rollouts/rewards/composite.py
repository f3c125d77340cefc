"""Reward composition (``src/forgeline/rollouts/rewards/composite.py`` contract):
verifier adapters, tag-format bonus, weighted composites with optional clip,
callables, and ``score_trajectories`` which rejects non-finite rewards with
``InvalidRewardError`` and uses a provider's ``score_many`` when it has one."""

from __future__ import annotations

import math
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

from rl_project_b200.core.errors import InvalidRewardError
from rl_project_b200.core.protocols import RewardProvider, RewardResult, Trajectory, Verifier
from rl_project_b200.rollouts.verifiers import tag_format_reward


def _finite(value: Any, source: str) -> float:
    if value is None or not isinstance(value, (int, float)) or not math.isfinite(float(value)):
        raise InvalidRewardError(f"reward provider {source!r} returned non-finite value {value!r}")
    return float(value)


class VerifierReward:
    def __init__(self, verifier: Verifier, target_key: str = "answer", weight: float = 1.0, on_tokens: bool = False):
        self.verifier = verifier
        self.target_key = target_key
        self.weight = weight
        self.on_tokens = on_tokens or getattr(verifier, "name", "") == "last_token_parity"
        self.name = f"verifier:{verifier.name}"

    def score(self, trajectory: Trajectory) -> RewardResult:
        output = trajectory.response_ids if self.on_tokens else trajectory.response_text
        res = self.verifier.verify(output, trajectory.task.get(self.target_key))
        return RewardResult(_finite(res.value, self.name) * self.weight, passed=res.passed,
                            components={self.name: res.value}, info=res.info)

    def score_many(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        return [self.score(t) for t in trajectories]


class TagFormatReward:
    name = "tag_format"

    def score(self, trajectory: Trajectory) -> RewardResult:
        return RewardResult(tag_format_reward(trajectory.response_text))


class CompositeReward:
    def __init__(self, providers: Sequence[Tuple[RewardProvider, float]], name: str = "composite",
                 clip: Optional[Tuple[float, float]] = None):
        if not providers:
            raise InvalidRewardError("composite reward needs at least one provider")
        self.providers = list(providers)
        self.name = name
        self.clip = clip

    def score(self, trajectory: Trajectory) -> RewardResult:
        total, comps, passed, info = 0.0, {}, None, {}
        for prov, w in self.providers:
            r = prov.score(trajectory)
            v = _finite(r.value, prov.name)
            comps[prov.name] = v
            total += w * v
            if passed is None and r.passed is not None:
                passed = r.passed
            if r.info:
                info[prov.name] = r.info
        if self.clip is not None:
            total = min(max(total, self.clip[0]), self.clip[1])
        return RewardResult(total, components=comps, passed=passed, info=info)


class CallableReward:
    def __init__(self, fn: Callable[[Trajectory], float], name: str = "callable"):
        self.fn = fn
        self.name = name

    def score(self, trajectory: Trajectory) -> RewardResult:
        return RewardResult(_finite(self.fn(trajectory), self.name))


def score_trajectories(provider: RewardProvider, trajectories: List[Trajectory]) -> List[float]:
    many = getattr(provider, "score_many", None)
    results = many(trajectories) if callable(many) else [provider.score(t) for t in trajectories]
    out = []
    for t, r in zip(trajectories, results):
        _finite(r.value, provider.name)
        t.reward = r
        out.append(r.value)
    return out
