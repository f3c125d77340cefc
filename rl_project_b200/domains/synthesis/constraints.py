"""Feasible ranges and defaults of generated synthesis conditions.

The four condition keys, their bounds and defaults are those of
``src/forgeline/domains/synthesis/constraints.py:8-20`` (they define the record
format and which generated conditions count as valid)."""

from __future__ import annotations

import math
from typing import Any, Dict, List, Tuple

CONDITION_BOUNDS: Dict[str, Tuple[float, float]] = {
    "temperature_celsius": (0.0, 300.0),
    "time_hours": (0.25, 48.0),
    "catalyst_loading_M": (0.001, 1.0),
    "solvent_ratio_ml_mmol": (0.5, 20.0),
}
CONDITION_DEFAULTS: Dict[str, float] = {"temperature_celsius": 80.0, "time_hours": 4.0, "catalyst_loading_M": 0.05,
                                        "solvent_ratio_ml_mmol": 3.0}


def validate_conditions(conditions: Dict[str, Any]) -> Tuple[Dict[str, Any], bool]:
    """Clip every condition into its range; ``valid`` is False if any was missing, non-numeric, NaN or clipped."""
    out = dict(conditions)
    valid = True
    for key, (lo, hi) in CONDITION_BOUNDS.items():
        try:
            v = float(conditions[key])
        except (KeyError, TypeError, ValueError):
            out[key], valid = CONDITION_DEFAULTS[key], False
            continue
        if math.isnan(v):
            out[key], valid = CONDITION_DEFAULTS[key], False
        elif not lo <= v <= hi:
            out[key], valid = min(hi, max(lo, v)), False
    return out, valid


def batch_validate(conditions_list: List[Dict[str, Any]]):
    pairs = [validate_conditions(c) for c in conditions_list]
    return [p[0] for p in pairs], [p[1] for p in pairs]


def validity_penalty(was_valid: bool, penalty: float = 0.05) -> float:
    return 0.0 if was_valid else -penalty
