"""Regression rules: compare a candidate's metrics with a baseline's.

Fail-closed semantics of ``src/forgeline/evaluation/regression.py:11-65``: a
missing or non-finite metric on either side fails its check, and an empty rule
list never passes.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Mapping, Optional

DIRECTIONS = ("higher_is_better", "lower_is_better")


@dataclass
class RegressionRule:
    metric: str
    direction: str = "higher_is_better"
    max_regression: float = 0.0  # allowed worsening (absolute, or a fraction of |baseline| if relative)
    relative: bool = False

    def validate(self) -> None:
        if self.direction not in DIRECTIONS:
            raise ValueError(f"direction must be one of {DIRECTIONS}")
        if self.max_regression < 0:
            raise ValueError("max_regression must be >= 0")


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


def _finite(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(float(v))


def _check(rule: RegressionRule, c, b) -> RegressionCheck:
    if not _finite(c):
        return RegressionCheck(rule.metric, False, c, b, "candidate metric missing or non-finite")
    if not _finite(b):
        return RegressionCheck(rule.metric, False, c, b, "baseline metric missing or non-finite")
    slack = rule.max_regression * (abs(b) if rule.relative else 1.0)
    if rule.direction == "higher_is_better":
        bound, ok, op = b - slack, c >= b - slack, ">="
    else:
        bound, ok, op = b + slack, c <= b + slack, "<="
    verdict = "ok" if ok else "regressed"
    return RegressionCheck(rule.metric, ok, c, b, f"{verdict}: need {op} {bound:.6g}, got {c:.6g}")


def evaluate_regression(candidate: Mapping[str, float], baseline: Mapping[str, float],
                        rules: List[RegressionRule]) -> RegressionReport:
    for r in rules:
        r.validate()
    checks = [_check(r, candidate.get(r.metric), baseline.get(r.metric)) for r in rules]
    return RegressionReport(passed=bool(rules) and all(c.passed for c in checks), checks=checks)
