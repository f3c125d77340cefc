"""Rule-based synthesis reward.

score = 0.40 yield + 0.30 selectivity + 0.20 (1 - safety risk) + 0.10 / (1 + steps / 10),
clipped to [0, 1] -- the weights of ``src/forgeline/domains/synthesis/reward.py:10-36``,
kept so scores of recorded runs compare across frameworks.
"""

from __future__ import annotations

from typing import Any, Dict, List

from rl_project_b200.core.protocols import RewardResult, Trajectory
from rl_project_b200.domains.synthesis.prompts import decode_conditions

RULE_WEIGHTS = {"yield": 0.40, "selectivity": 0.30, "safety": 0.20, "efficiency": 0.10}

_FIELDS = (("yield", "outcomes", "yield", 0.5), ("selectivity", "outcomes", "selectivity", 0.5),
           ("safety_risk", "outcomes", "safety_risk", 0.5), ("steps", "outcomes", "steps", 5.0),
           ("temperature", "parameters", "temperature_celsius", 80.0), ("time", "parameters", "time_hours", 4.0),
           ("catalyst", "parameters", "catalyst_loading_M", 0.05),
           ("solvent", "parameters", "solvent_ratio_ml_mmol", 3.0))


def extract_outcomes(traj: Dict[str, Any]) -> Dict[str, float]:
    """Flat view of a record whose fields sit at the top level or under ``outcomes`` / ``parameters``."""
    out = {}
    for name, section, key, default in _FIELDS:
        nested = traj.get(section) or {}
        out[name] = float(nested.get(key, traj.get(key, default)))
    return out


def rule_score(traj: Dict[str, Any]) -> float:
    o = extract_outcomes(traj)
    w = RULE_WEIGHTS
    s = (w["yield"] * o["yield"] + w["selectivity"] * o["selectivity"] + w["safety"] * (1.0 - o["safety_risk"])
         + w["efficiency"] / (1.0 + o["steps"] / 10.0))
    return float(min(1.0, max(0.0, s)))


def trajectory_to_text(traj: Dict[str, Any]) -> str:
    o = extract_outcomes(traj)
    return (f"{traj.get('molecule', 'compound')}: {o['temperature']:.0f} C for {o['time']:.1f} h, catalyst "
            f"{o['catalyst']:.3f} M, solvent {o['solvent']:.1f} mL/mmol -> yield {o['yield']:.2f}, selectivity "
            f"{o['selectivity']:.2f}, risk {o['safety_risk']:.2f}, {int(o['steps'])} steps")


class SynthesisRuleReward:
    """Scores a trajectory whose ``task`` is the synthesis record; conditions decoded from the
    generated JSON are merged in first (``passed`` at score >= 0.75)."""

    name = "synthesis_rule"

    def __init__(self, decode_from_text: bool = True):
        self.decode_from_text = decode_from_text

    def score_record(self, record: Dict[str, Any]) -> float:
        return rule_score(record)

    def score_batch(self, records: List[Dict[str, Any]]) -> List[float]:
        return [rule_score(r) for r in records]

    def score(self, trajectory: Trajectory) -> RewardResult:
        record = dict(trajectory.task)
        valid = True
        if self.decode_from_text and trajectory.response_text:
            cond, valid = decode_conditions(trajectory.response_text)
            record.update(cond)
        value = rule_score(record)
        return RewardResult(value=value, passed=value >= 0.75, components={"rule": value},
                            info={"conditions_valid": valid})
