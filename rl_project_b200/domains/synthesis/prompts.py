"""Prompt template and JSON codec of synthesis conditions."""

from __future__ import annotations

import json
import re
from typing import Any, Dict, Tuple

from rl_project_b200.domains.synthesis.constraints import CONDITION_DEFAULTS, validate_conditions

CONDITION_KEYS = ("temperature_celsius", "time_hours", "catalyst_loading_M", "solvent_ratio_ml_mmol")

PROMPT_TEMPLATE = ("### Task: propose synthesis conditions\n"
                   "Target molecule: {molecule} (CAS {cas})\n"
                   "Goal: high yield and selectivity, low hazard, few steps.\n"
                   "### Conditions as JSON:\n")

_JSON_OBJ = re.compile(r"\{[^{}]*\}", re.DOTALL)


def build_synthesis_prompt(record: Dict[str, Any]) -> str:
    return PROMPT_TEMPLATE.format(molecule=record.get("molecule", "Unknown"), cas=record.get("cas_number", "N/A"))


def conditions_to_json(record: Dict[str, Any]) -> str:
    params = record.get("parameters", record)
    return json.dumps({k: params.get(k, record.get(k, CONDITION_DEFAULTS[k])) for k in CONDITION_KEYS})


def decode_conditions(text: str) -> Tuple[Dict[str, Any], bool]:
    """First JSON object in ``text`` (defaults when none parses), clipped to the feasible ranges."""
    for m in _JSON_OBJ.finditer(text or ""):
        try:
            raw = json.loads(m.group())
        except json.JSONDecodeError:
            continue
        if isinstance(raw, dict):
            return validate_conditions(raw)
    return validate_conditions(dict(CONDITION_DEFAULTS))[0], False
