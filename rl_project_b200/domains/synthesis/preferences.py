"""Preference pairs and SFT records built from synthesis trajectories."""

from __future__ import annotations

import random
from typing import Any, Dict, List, Tuple

from rl_project_b200.data.records import PreferenceRecord, SFTRecord
from rl_project_b200.domains.synthesis.prompts import build_synthesis_prompt, conditions_to_json
from rl_project_b200.domains.synthesis.reward import extract_outcomes, rule_score


def _yield(t: Dict[str, Any]) -> float:
    return extract_outcomes(t)["yield"]


def build_preference_pairs(trajectories: List[Dict[str, Any]], pairs_per_molecule: int = 20,
                           seed: int = 0) -> List[Tuple[Dict, Dict]]:
    """Per molecule, pair a run from the better-yield half with one from the worse half (seeded)."""
    rng = random.Random(seed)
    groups: Dict[str, List[Dict]] = {}
    for t in trajectories:
        groups.setdefault(t.get("molecule", "unknown"), []).append(t)
    pairs: List[Tuple[Dict, Dict]] = []
    for runs in groups.values():
        if len(runs) < 2:
            continue
        ranked = sorted(runs, key=_yield, reverse=True)
        half = len(ranked) // 2
        better, worse = ranked[:half], ranked[half:]
        pairs.extend((rng.choice(better), rng.choice(worse)) for _ in range(pairs_per_molecule))
    return pairs


def pairs_to_records(pairs: List[Tuple[Dict, Dict]]) -> List[PreferenceRecord]:
    out = []
    for chosen, rejected in pairs:
        c, r = conditions_to_json(chosen), conditions_to_json(rejected)
        if c != r:
            out.append(PreferenceRecord(prompt=build_synthesis_prompt(chosen), chosen=c, rejected=r,
                                        meta={"molecule": chosen.get("molecule"), "chosen_yield": _yield(chosen),
                                              "rejected_yield": _yield(rejected)}))
    return out


def filter_high_reward(trajectories: List[Dict[str, Any]], threshold: float) -> List[Dict[str, Any]]:
    return [t for t in trajectories if rule_score(t) >= threshold]


def build_sft_records(trajectories: List[Dict[str, Any]]) -> List[SFTRecord]:
    return [SFTRecord(prompt=build_synthesis_prompt(t), response=conditions_to_json(t),
                      meta={"molecule": t.get("molecule")}) for t in trajectories]
