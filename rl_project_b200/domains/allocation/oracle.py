"""Hindsight upper bound: the best expected value with the whole opportunity stream
known in advance and the (policy-dependent) pressure switched off.

Without pressure the problem is a concave resource allocation: maximise
sum_t v_t q_t (1 - e^{-u_t}) subject to sum_t u_t c_t <= B, 0 <= u_t <= u_max.
The KKT conditions give u_t(lambda) = clip(ln(v_t q_t / (lambda c_t)), 0, u_max);
the price lambda is found by bisection on the budget.  A valid upper bound for
every policy, because pressure only raises costs and lowers response rates.
"""

from __future__ import annotations

from typing import Dict, List, Sequence

import numpy as np

from rl_project_b200.domains.allocation.env import AllocationEnvConfig, Opportunity, draw_episode


def hindsight_upper_bound(opps: Sequence[Opportunity], budget: float, u_max: float) -> Dict[str, float]:
    a = np.array([o.value * o.quality for o in opps])
    c = np.array([o.cost for o in opps])

    def alloc(lam: float) -> np.ndarray:
        with np.errstate(divide="ignore"):
            return np.clip(np.log(np.maximum(a, 1e-300) / (lam * c)), 0.0, u_max)

    if float((u_max * c).sum()) <= budget:
        u = np.full(len(a), u_max)
    else:
        lo, hi = 1e-12, float((a / c).max()) + 1.0
        for _ in range(100):
            mid = 0.5 * (lo + hi)
            if float((alloc(mid) * c).sum()) > budget:
                lo = mid
            else:
                hi = mid
        u = alloc(hi)
    return {"value": float((a * (1.0 - np.exp(-u))).sum()), "spend": float((u * c).sum()),
            "mean_intensity": float(u.mean())}


def oracle_for_seed(env_cfg: AllocationEnvConfig, seed: int) -> Dict[str, float]:
    ep = draw_episode(env_cfg, seed)
    opps: List[Opportunity] = [Opportunity(float(v), float(c), float(q), float(s)) for v, c, q, s in
                               zip(ep["value"], ep["cost"], ep["quality"], ep["season"])]
    return hindsight_upper_bound(opps, env_cfg.budget, max(env_cfg.multipliers))


def oracle_values(env_cfg: AllocationEnvConfig, seeds: Sequence[int]) -> np.ndarray:
    return np.array([oracle_for_seed(env_cfg, int(s))["value"] for s in seeds])
