"""Regression gates: a candidate's metrics against a baseline's (the rule / check / report types and the
fail-closed semantics of ``src/forgeline/evaluation/regression.py``: a missing or non-finite metric on
either side fails its check, and an empty rule list never passes).

A rule's direction is a sign: with ``s = +1`` for higher-is-better and ``-1`` for lower-is-better, a check
passes when ``s * (candidate - baseline) >= -slack``, where the slack is ``max_regression`` (times
``|baseline|`` for relative rules).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Mapping, Optional

_SIGN = {"higher_is_better": 1.0, "lower_is_better": -1.0}
DIRECTIONS = tuple(_SIGN)


@dataclass
class RegressionRule:
    metric: str
    direction: str = "higher_is_better"
    max_regression: float = 0.0  # allowed worsening: absolute, or a fraction of |baseline| when relative
    relative: bool = False

    def validate(self) -> None:
        if self.direction not in _SIGN:
            raise ValueError(f"direction must be one of {DIRECTIONS}")
        if self.max_regression < 0:
            raise ValueError("max_regression must be >= 0")

    def slack(self, baseline: float) -> float:
        return self.max_regression * (abs(baseline) if self.relative else 1.0)


@dataclass
class RegressionCheck:
    metric: str
    passed: bool
    candidate: Optional[float]
    baseline: Optional[float]
    reason: str


@dataclass
class RegressionReport:
    passed: bool
    checks: List[RegressionCheck] = field(default_factory=list)

    def failures(self) -> List[RegressionCheck]:
        return [c for c in self.checks if not c.passed]


def _usable(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(float(v))


def _check(rule: RegressionRule, cand, base) -> RegressionCheck:
    for side, v in (("candidate", cand), ("baseline", base)):
        if not _usable(v):
            return RegressionCheck(rule.metric, False, cand, base, f"{side} metric missing or non-finite")
    sign, slack = _SIGN[rule.direction], rule.slack(base)
    ok = sign * (cand - base) >= -slack
    limit = base - sign * slack
    word = "ok" if ok else "regressed"
    return RegressionCheck(rule.metric, ok, cand, base,
                           f"{word}: need {'>=' if sign > 0 else '<='} {limit:.6g}, got {cand:.6g}")


def evaluate_regression(candidate: Mapping[str, float], baseline: Mapping[str, float],
                        rules: List[RegressionRule]) -> RegressionReport:
    for rule in rules:
        rule.validate()
    checks = [_check(rule, candidate.get(rule.metric), baseline.get(rule.metric)) for rule in rules]
    return RegressionReport(passed=bool(checks) and all(c.passed for c in checks), checks=checks)
