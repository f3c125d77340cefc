"""Feasible ranges and defaults of generated synthesis conditions.

The four condition keys, their bounds and defaults are those of
``src/forgeline/domains/synthesis/constraints.py:8-20`` (they define the record
format and which generated conditions count as valid)."""

from __future__ import annotations

import math
from typing import Any, Dict, List, Tuple

import numpy as np

CONDITION_BOUNDS: Dict[str, Tuple[float, float]] = {
    "temperature_celsius": (0.0, 300.0),
    "time_hours": (0.25, 48.0),
    "catalyst_loading_M": (0.001, 1.0),
    "solvent_ratio_ml_mmol": (0.5, 20.0),
}
CONDITION_DEFAULTS: Dict[str, float] = {"temperature_celsius": 80.0, "time_hours": 4.0, "catalyst_loading_M": 0.05,
                                        "solvent_ratio_ml_mmol": 3.0}


def _as_float(v: Any) -> float:
    try:
        return float(v)
    except (TypeError, ValueError):
        return math.nan


def batch_validate(conditions_list: List[Dict[str, Any]]):
    """``(clipped, valid)`` for every record, computed column-wise over one ``[records, 4]`` array: a missing,
    non-numeric or NaN value takes its default, an out-of-range one is clipped, and either makes the record
    invalid."""
    keys = list(CONDITION_BOUNDS)
    raw = np.array([[_as_float(c.get(k)) for k in keys] for c in conditions_list], dtype=np.float64).reshape(-1, 4)
    lo = np.array([CONDITION_BOUNDS[k][0] for k in keys])
    hi = np.array([CONDITION_BOUNDS[k][1] for k in keys])
    default = np.array([CONDITION_DEFAULTS[k] for k in keys])
    missing = np.isnan(raw)
    fixed = np.where(missing, default, np.clip(raw, lo, hi))
    valid = ~(missing | (raw < lo) | (raw > hi)).any(axis=1)
    clipped = [{**c, **dict(zip(keys, row.tolist()))} for c, row in zip(conditions_list, fixed)]
    return clipped, valid.tolist()


def validate_conditions(conditions: Dict[str, Any]) -> Tuple[Dict[str, Any], bool]:
    """Clip every condition into its range; ``valid`` is False if any was missing, non-numeric, NaN or clipped."""
    clipped, valid = batch_validate([conditions])
    return clipped[0], valid[0]


def validity_penalty(was_valid: bool, penalty: float = 0.05) -> float:
    return 0.0 if was_valid else -penalty
