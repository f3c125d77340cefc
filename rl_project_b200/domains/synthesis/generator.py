"""Seeded simulator of synthesis runs with chemistry-shaped response surfaces.

Each molecule has an optimum (temperature, time, catalyst and solvent windows,
best yield).  Yield falls off as a Gaussian in temperature, saturates then
slowly degrades in time (over-reaction), and has soft windows in catalyst
loading and solvent ratio; selectivity follows yield, hazard grows with
temperature and time.  ``predict_outcomes`` is the noise-free surface (used to
score generated conditions); ``simulate_trajectory`` samples conditions around
the optimum and adds measurement noise.  The molecule table holds public facts
(names, CAS numbers, molar masses) plus this simulator's optima.
"""

from __future__ import annotations

import math
import random
from typing import Any, Dict, List, Optional

MOLECULES: Dict[str, Dict[str, Any]] = {
    "Aspirin": {"name": "Acetylsalicylic acid", "cas": "50-78-2", "molar_mass": 180.16,
                "best_yield": 0.94, "t_opt": 85.0, "h_opt": 2.0},
    "Ibuprofen": {"name": "2-(4-isobutylphenyl)propanoic acid", "cas": "15687-27-1", "molar_mass": 206.29,
                  "best_yield": 0.87, "t_opt": 105.0, "h_opt": 4.0},
    "Paracetamol": {"name": "N-(4-hydroxyphenyl)acetamide", "cas": "103-90-2", "molar_mass": 151.16,
                    "best_yield": 0.91, "t_opt": 75.0, "h_opt": 2.5},
    "Naproxen": {"name": "(S)-6-methoxy-alpha-methyl-2-naphthaleneacetic acid", "cas": "22204-53-1",
                 "molar_mass": 230.26, "best_yield": 0.78, "t_opt": 120.0, "h_opt": 6.0},
    "Ketoprofen": {"name": "2-(3-benzoylphenyl)propanoic acid", "cas": "22071-15-4", "molar_mass": 254.28,
                   "best_yield": 0.83, "t_opt": 100.0, "h_opt": 4.5},
}


def _window(x: float, lo: float, hi: float, width: float) -> float:
    """1 inside [lo, hi], decaying smoothly (Gaussian shoulders of ``width``) outside."""
    d = lo - x if x < lo else x - hi if x > hi else 0.0
    return math.exp(-(d / width) ** 2)


def predict_outcomes(molecule: str, conditions: Dict[str, float]) -> Dict[str, float]:
    m = MOLECULES.get(molecule)
    if m is None:
        return {"yield": 0.5, "selectivity": 0.5, "safety_risk": 0.5, "steps": 5.0}
    t = float(conditions.get("temperature_celsius", 80.0))
    h = float(conditions.get("time_hours", 4.0))
    cat = float(conditions.get("catalyst_loading_M", 0.05))
    sol = float(conditions.get("solvent_ratio_ml_mmol", 3.0))
    f_temp = math.exp(-((t - m["t_opt"]) / 28.0) ** 2)
    f_time = (1.0 - math.exp(-2.5 * h / m["h_opt"])) / (1.0 - math.exp(-2.5)) * \
        (1.0 / (1.0 + 0.08 * max(0.0, h - 1.8 * m["h_opt"])))
    f_cat = 0.45 + 0.55 * _window(cat, 0.05, 0.15, 0.06)
    f_sol = 0.55 + 0.45 * _window(sol, 1.0, 3.0, 1.5)
    y = min(0.97, max(0.05, m["best_yield"] * min(1.0, f_time) * f_temp * f_cat * f_sol))
    return {"yield": y, "selectivity": min(0.98, 0.62 + 0.36 * y),
            "safety_risk": min(0.9, 0.08 + 0.0025 * max(0.0, t - 70.0) + 0.012 * max(0.0, h - 4.0)),
            "steps": 3.0 + (2.0 if h > 8.0 else 0.0)}


def simulate_trajectory(molecule: str, idx: int, rng: random.Random) -> Dict[str, Any]:
    m = MOLECULES[molecule]
    cond = {"temperature_celsius": round(min(160.0, max(25.0, rng.gauss(m["t_opt"], 25.0))), 1),
            "time_hours": round(min(14.0, max(0.5, m["h_opt"] * math.exp(rng.gauss(0.0, 0.45)))), 2),
            "catalyst_loading_M": round(math.exp(rng.uniform(math.log(0.01), math.log(0.35))), 3),
            "solvent_ratio_ml_mmol": round(rng.uniform(0.5, 6.5), 2)}
    o = predict_outcomes(molecule, cond)
    y = min(0.97, max(0.05, o["yield"] * rng.gauss(1.0, 0.06)))
    return {"molecule": molecule, "cas_number": m["cas"], "molar_mass": m["molar_mass"], "procedure_id": idx,
            "procedure": f"Synthesis of {m['name']}",
            "parameters": {**cond, "hazards": ["thermal" if cond["temperature_celsius"] > 100 else "none",
                                               "long" if cond["time_hours"] > 6 else "normal"]},
            "outcomes": {"yield": round(y, 3), "selectivity": round(min(0.98, 0.62 + 0.36 * y), 3),
                         "safety_risk": round(o["safety_risk"], 3), "steps": int(o["steps"]),
                         "molar_mass_product": m["molar_mass"]},
            "data_source": "simulated"}


def simulate_dataset(per_molecule: int = 100, seed: int = 0, molecules: Optional[List[str]] = None) -> List[Dict]:
    rng = random.Random(seed)
    return [simulate_trajectory(mol, i, rng) for mol in (molecules or list(MOLECULES)) for i in range(per_molecule)]


def yield_series_trajectories(seed: int = 0, points: int = 10) -> List[Dict]:
    """Per molecule, conditions swept from far below to the optimum (a rising yield series)."""
    rng = random.Random(seed)
    out = []
    for mol, m in MOLECULES.items():
        for i in range(points):
            frac = i / max(points - 1, 1)
            cond = {"temperature_celsius": round(m["t_opt"] - 45.0 * (1.0 - frac), 1),
                    "time_hours": round(max(0.5, m["h_opt"] * (0.35 + 0.65 * frac)), 2),
                    "catalyst_loading_M": round(0.1 + rng.gauss(0.0, 0.01), 3),
                    "solvent_ratio_ml_mmol": round(2.0 + rng.gauss(0.0, 0.2), 2)}
            o = predict_outcomes(mol, cond)
            out.append({"molecule": mol, "cas_number": m["cas"], "procedure_id": i, "parameters": cond,
                        "outcomes": {k: round(v, 3) for k, v in o.items()}})
    return out
