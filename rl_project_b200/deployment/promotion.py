"""Fail-closed promotion gates.

A ``PromotionGate`` holds ``GateRule`` s over candidate metrics (absolute
``min`` / ``max``) and, optionally, over the incumbent's (``min_delta`` /
``max_increase``, absolute or relative).  A candidate passes only when every
rule passes; a missing or non-finite metric fails its rule.  With
``when_no_baseline="skip_relative"`` the relative rules are skipped when there
is no incumbent at all (the first promotion); absolute rules always apply.
Semantics of ``src/forgeline/deployment/promotion.py:20-128``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any, Dict, List, Mapping, Optional

from rl_project_b200.core.errors import ConfigError, PromotionError


@dataclass
class GateRule:
    metric: str
    min: Optional[float] = None
    max: Optional[float] = None
    min_delta: Optional[float] = None
    max_increase: Optional[float] = None
    relative: bool = False
    description: str = ""

    def validate(self) -> None:
        if self.min is None and self.max is None and self.min_delta is None and self.max_increase is None:
            raise ConfigError(f"gate rule for {self.metric!r} has no constraint")
        if self.min is not None and self.max is not None and self.min > self.max:
            raise ConfigError(f"gate rule for {self.metric!r}: min > max")

    @property
    def needs_baseline(self) -> bool:
        return self.min_delta is not None or self.max_increase is not None

    @classmethod
    def from_dict(cls, d: Mapping[str, Any]) -> "GateRule":
        unknown = set(d) - set(cls.__dataclass_fields__)
        if unknown:
            raise ConfigError(f"unknown gate rule keys: {sorted(unknown)}")
        rule = cls(**dict(d))
        rule.validate()
        return rule


@dataclass
class GateCheck:
    metric: str
    passed: bool
    candidate: Optional[float]
    baseline: Optional[float]
    reason: str


@dataclass
class PromotionReport:
    passed: bool
    checks: List[GateCheck] = field(default_factory=list)

    def failures(self) -> List[GateCheck]:
        return [c for c in self.checks if not c.passed]

    def to_dict(self) -> Dict[str, Any]:
        return {"passed": self.passed, "checks": [dict(c.__dict__) for c in self.checks]}


def _finite(v: Any) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(float(v))


class PromotionGate:
    def __init__(self, rules: List[GateRule], require_baseline: bool = False, when_no_baseline: str = "fail"):
        if not rules:
            raise ConfigError("promotion gate needs at least one rule")
        if when_no_baseline not in ("fail", "skip_relative"):
            raise ConfigError("when_no_baseline must be 'fail' or 'skip_relative'")
        for r in rules:
            r.validate()
        self.rules = list(rules)
        self.require_baseline = require_baseline
        self.when_no_baseline = when_no_baseline

    @classmethod
    def from_config(cls, config: Mapping[str, Any]) -> "PromotionGate":
        rules = config.get("rules")
        if not isinstance(rules, list) or not rules:
            raise ConfigError("promotion config needs a non-empty 'rules' list")
        return cls([GateRule.from_dict(r) for r in rules], require_baseline=bool(config.get("require_baseline", False)),
                   when_no_baseline=str(config.get("when_no_baseline", "fail")))

    def _check(self, rule: GateRule, candidate: Mapping[str, float],
               baseline: Optional[Mapping[str, float]]) -> GateCheck:
        c = candidate.get(rule.metric)
        b = baseline.get(rule.metric) if baseline is not None else None
        if not _finite(c):
            return GateCheck(rule.metric, False, None if c is None else float("nan"), b,
                             "candidate metric missing or non-finite")
        c = float(c)
        # (active, violated, message) of every absolute bound
        bounds = [(rule.min is not None, lambda: c < rule.min, lambda: f"{c:.6g} < min {rule.min:.6g}"),
                  (rule.max is not None, lambda: c > rule.max, lambda: f"{c:.6g} > max {rule.max:.6g}")]
        problems = [msg() for active, bad, msg in bounds if active and bad()]
        note = ""
        if rule.needs_baseline:
            if baseline is None and self.when_no_baseline == "skip_relative":
                return GateCheck(rule.metric, not problems, c, None,
                                 ("; ".join(problems) or "ok") + " (relative rule skipped: no incumbent)")
            if not _finite(b):
                return GateCheck(rule.metric, False, c, b, "baseline metric missing or non-finite")
            b = float(b)
            scale = abs(b) if rule.relative else 1.0
            relative = [(rule.min_delta, lambda d: c < b + d, lambda d: f"{c:.6g} < baseline {b:.6g} + {d:.6g}"),
                        (rule.max_increase, lambda d: c > b + d, lambda d: f"{c:.6g} > baseline {b:.6g} + {d:.6g}")]
            problems += [msg(v * scale) for v, bad, msg in relative if v is not None and bad(v * scale)]
        return GateCheck(rule.metric, not problems, c, b, ("; ".join(problems) or "ok") + note)

    def evaluate(self, candidate: Mapping[str, float],
                 baseline: Optional[Mapping[str, float]] = None) -> PromotionReport:
        if self.require_baseline and baseline is None:
            return PromotionReport(False, [GateCheck("*", False, None, None, "baseline metrics required but missing")])
        checks = [self._check(r, candidate, baseline) for r in self.rules]
        return PromotionReport(passed=all(c.passed for c in checks), checks=checks)

    def assert_promotable(self, candidate: Mapping[str, float],
                          baseline: Optional[Mapping[str, float]] = None) -> PromotionReport:
        report = self.evaluate(candidate, baseline)
        if not report.passed:
            failing = ", ".join(f"{c.metric} ({c.reason})" for c in report.failures())
            raise PromotionError(f"promotion rejected: {failing}")
        return report
