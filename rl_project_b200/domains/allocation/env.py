"""Budgeted sequential allocation: a finite-horizon, budget-constrained POMDP.

The decision problem, its parameters and the 14-feature observation are those
of ``src/forgeline/domains/allocation/env.py:1-60`` (the config keys and the
observation layout are part of the domain's interface: logged episodes and
trained policies carry them).  Per step, for opportunity (value v, base cost
c, quality q, season s) and action a with multiplier m = M[a]:

    effective cost  c' = c (1 + kappa p)         p = latent pressure (not observed)
    spend           x = min(m c', remaining)      (a clipped request is a violation)
    intensity       u = x / c'
    response rate   rho = q (1 - e^-u) max(0, 1 - phi p)
    outcome         y ~ Bernoulli(rho) (pre-drawn uniforms), reward = y v
    pressure        p <- delta p + eta u

This implementation is vectorised: ``VectorEnv`` steps ``n`` episodes as numpy
arrays in lockstep (every policy acts on a batch); ``BudgetedAllocationEnv`` is
the single-episode view of the same arrays.
"""

from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Mapping, Optional, Sequence, Tuple

import numpy as np

from rl_project_b200.core.errors import ConfigError

MULTIPLIERS: Tuple[float, ...] = (0.0, 0.5, 1.0, 1.5)
ACTION_NAMES: Tuple[str, ...] = ("abstain", "low", "medium", "high")
OBS_DIM = 14
OBS_NAMES: Tuple[str, ...] = ("remaining_frac", "elapsed_frac", "remaining_steps_frac", "value_rel", "cost_rel",
                              "quality", "season", "pacing_error", "cum_value_norm", "last_multiplier",
                              "last_reward_rel", "last_spend_rel", "recent_value_rel", "recent_cost_rel")


def strict_config(cls, data: Mapping[str, Any], what: str, coerce: Optional[Dict[str, Callable]] = None):
    """Build the dataclass ``cls`` from ``data``: unknown keys are a ``ConfigError`` naming ``what``, values
    of the keys in ``coerce`` go through their converter, and the result's ``validate()`` (if any) runs."""
    names = {f.name for f in dataclasses.fields(cls)}
    unknown = sorted(set(data) - names)
    if unknown:
        raise ConfigError(f"unknown {what} keys: {unknown}")
    conv = coerce or {}
    obj = cls(**{k: (conv[k](v) if k in conv else v) for k, v in data.items()})
    if hasattr(obj, "validate"):
        obj.validate()
    return obj


def response_gain(u):
    """Concave, saturating response to intensity: g(u) = 1 - exp(-u)."""
    return 1.0 - np.exp(-np.asarray(u, dtype=np.float64))


@dataclass
class AllocationEnvConfig:
    horizon: int = 48
    budget: float = 24.0
    value_mean: float = 1.0
    value_sigma: float = 0.5
    cost_mean: float = 1.0
    cost_sigma: float = 0.3
    quality_alpha: float = 2.0
    quality_beta: float = 2.0
    season_amplitude_value: float = 0.4
    season_amplitude_cost: float = -0.2
    random_phase: bool = True
    pressure_decay: float = 0.85
    pressure_gain: float = 0.25
    pressure_cost_coef: float = 0.6
    pressure_response_coef: float = 0.35
    history_window: int = 4
    multipliers: Tuple[float, ...] = MULTIPLIERS

    def validate(self) -> None:
        checks = [(self.horizon >= 2, "allocation env horizon must be >= 2"),
                  (min(self.budget, self.value_mean, self.cost_mean) > 0,
                   "budget, value_mean and cost_mean must be positive"),
                  (0.0 <= self.pressure_decay < 1.0, "pressure_decay must be in [0, 1)"),
                  (min(self.pressure_gain, self.pressure_cost_coef, self.pressure_response_coef) >= 0,
                   "pressure coefficients must be >= 0"),
                  (min(self.value_sigma, self.cost_sigma) >= 0 and min(self.quality_alpha, self.quality_beta) > 0,
                   "invalid opportunity distribution parameters"),
                  (len(self.multipliers) >= 2 and self.multipliers[0] == 0.0 and min(self.multipliers) >= 0,
                   "multipliers must start with 0 (abstain) and be non-negative"),
                  (self.history_window >= 1, "history_window must be >= 1")]
        for ok, msg in checks:
            if not ok:
                raise ConfigError(msg)

    @classmethod
    def from_dict(cls, data: Dict[str, Any]) -> "AllocationEnvConfig":
        return strict_config(cls, data, "allocation env",
                             coerce={"multipliers": lambda ms: tuple(float(m) for m in ms)})

    def to_dict(self) -> Dict[str, Any]:
        d = dataclasses.asdict(self)
        d["multipliers"] = list(self.multipliers)
        return d

    @property
    def n_actions(self) -> int:
        return len(self.multipliers)


@dataclass
class Opportunity:
    value: float
    cost: float
    quality: float
    season: float


@dataclass
class StepInfo:
    t: int
    action: int
    multiplier: float
    intensity: float
    effective_cost: float
    spend: float
    reward: float
    outcome: int
    response_rate: float
    pressure_before: float
    pressure_after: float
    remaining_before: float
    remaining_after: float
    clipped: bool
    opportunity: Opportunity


def draw_episode(cfg: AllocationEnvConfig, seed: Optional[int]) -> Dict[str, np.ndarray]:
    """The exogenous stream of one episode (values, costs, qualities, seasons, outcome uniforms)."""
    rng = np.random.default_rng(seed)
    T = cfg.horizon
    phase = rng.uniform(0, T) if cfg.random_phase else 0.0
    eps_v, eps_c = rng.standard_normal(T), rng.standard_normal(T)
    q = rng.beta(cfg.quality_alpha, cfg.quality_beta, size=T)
    u = rng.uniform(0.0, 1.0, size=T)
    s = np.sin(2.0 * math.pi * (np.arange(T) + phase) / T)
    v = cfg.value_mean * np.exp(cfg.value_sigma * eps_v - 0.5 * cfg.value_sigma ** 2) * (1 + cfg.season_amplitude_value * s)
    c = cfg.cost_mean * np.exp(cfg.cost_sigma * eps_c - 0.5 * cfg.cost_sigma ** 2) * (1 + cfg.season_amplitude_cost * s)
    return {"value": np.maximum(v, 1e-6), "cost": np.maximum(c, 1e-6), "quality": q, "season": s, "uniform": u}


class VectorEnv:
    """``n`` independent episodes stepped together; all state is ``[n]`` / ``[n, T]`` arrays."""

    def __init__(self, config: AllocationEnvConfig, n: int):
        if n < 1:
            raise ConfigError("VectorEnv needs n >= 1")
        config.validate()
        self.cfg, self.n = config, n
        self.M = np.asarray(config.multipliers, dtype=np.float64)
        self.t = 0
        self.done = True

    def reset(self, seeds: Sequence[int]) -> np.ndarray:
        if len(seeds) != self.n:
            raise ConfigError("one seed per environment is required")
        eps = [draw_episode(self.cfg, int(s)) for s in seeds]
        for k in ("value", "cost", "quality", "season", "uniform"):
            setattr(self, k, np.stack([e[k] for e in eps]))
        z = np.zeros(self.n)
        self.remaining = np.full(self.n, float(self.cfg.budget))
        self.pressure, self.cum_spend, self.cum_value = z.copy(), z.copy(), z.copy()
        self.last_mult, self.last_reward, self.last_spend = z.copy(), z.copy(), z.copy()
        self.t, self.done = 0, False
        return self.observation()

    def context(self) -> "StepArrays":
        t = self.t
        return StepArrays(t=t, horizon=self.cfg.horizon, remaining=self.remaining.copy(), budget=self.cfg.budget,
                          cum_spend=self.cum_spend.copy(), value=self.value[:, t].copy(), cost=self.cost[:, t].copy(),
                          quality=self.quality[:, t].copy())

    def observation(self) -> np.ndarray:
        cfg, t, T = self.cfg, self.t, self.cfg.horizon
        lo = max(0, t - cfg.history_window)
        if t > lo:
            rv = (self.value[:, lo:t] / cfg.value_mean - 1.0).mean(1)
            rc = (self.cost[:, lo:t] / cfg.cost_mean - 1.0).mean(1)
        else:
            rv = rc = np.zeros(self.n)
        cols = [self.remaining / cfg.budget, np.full(self.n, t / T), np.full(self.n, (T - t) / T),
                self.value[:, t] / cfg.value_mean - 1.0, self.cost[:, t] / cfg.cost_mean - 1.0, self.quality[:, t],
                self.season[:, t], self.cum_spend / cfg.budget - t / T, self.cum_value / (T * cfg.value_mean),
                self.last_mult / self.M.max(), self.last_reward / cfg.value_mean, self.last_spend / cfg.cost_mean, rv, rc]
        return np.stack(cols, 1).astype(np.float32)

    def step(self, actions: Sequence[int]):
        if self.done:
            raise ConfigError("episode is finished; call reset()")
        a = np.asarray(actions, dtype=np.int64)
        if a.shape != (self.n,) or a.min() < 0 or a.max() >= self.cfg.n_actions:
            raise ConfigError(f"actions must be {self.n} ints in 0..{self.cfg.n_actions - 1}")
        cfg, t = self.cfg, self.t
        m = self.M[a]
        eff = self.cost[:, t] * (1.0 + cfg.pressure_cost_coef * self.pressure)
        requested = m * eff
        spend = np.minimum(requested, self.remaining)
        clipped = requested > self.remaining + 1e-12
        u = spend / eff
        rate = self.quality[:, t] * response_gain(u) * np.maximum(0.0, 1.0 - cfg.pressure_response_coef * self.pressure)
        outcome = (self.uniform[:, t] < rate).astype(np.int64)
        reward = outcome * self.value[:, t]
        p0, r0 = self.pressure.copy(), self.remaining.copy()
        self.pressure = cfg.pressure_decay * self.pressure + cfg.pressure_gain * u
        self.remaining = self.remaining - spend
        self.cum_spend += spend
        self.cum_value += reward
        self.last_mult, self.last_reward, self.last_spend = m, reward, spend
        infos = [StepInfo(t, int(a[i]), float(m[i]), float(u[i]), float(eff[i]), float(spend[i]), float(reward[i]),
                          int(outcome[i]), float(rate[i]), float(p0[i]), float(self.pressure[i]), float(r0[i]),
                          float(self.remaining[i]), bool(clipped[i]),
                          Opportunity(float(self.value[i, t]), float(self.cost[i, t]), float(self.quality[i, t]),
                                      float(self.season[i, t]))) for i in range(self.n)]
        self.t += 1
        self.done = self.t >= cfg.horizon
        obs = self.observation() if not self.done else np.zeros((self.n, OBS_DIM), dtype=np.float32)
        return obs, reward, np.full(self.n, self.done), infos


@dataclass
class StepArrays:
    """Raw (unnormalised) per-step quantities a policy may use, one entry per episode."""

    t: int
    horizon: int
    remaining: np.ndarray
    budget: float
    cum_spend: np.ndarray
    value: np.ndarray
    cost: np.ndarray
    quality: np.ndarray


@dataclass
class StepContext:
    """One episode's raw per-step scalars (``src/forgeline/domains/allocation/policies.py:41-51`` fields);
    ``StepArrays`` holds the same for a batch of episodes."""

    t: int
    horizon: int
    remaining: float
    budget: float
    cum_spend: float
    value: float
    cost: float
    quality: float

    @classmethod
    def from_arrays(cls, a: "StepArrays", i: int = 0) -> "StepContext":
        return cls(a.t, a.horizon, float(a.remaining[i]), float(a.budget), float(a.cum_spend[i]),
                   float(a.value[i]), float(a.cost[i]), float(a.quality[i]))

    def to_arrays(self) -> "StepArrays":
        one = lambda v: np.asarray([v], dtype=np.float64)  # noqa: E731
        return StepArrays(self.t, self.horizon, one(self.remaining), self.budget, one(self.cum_spend),
                          one(self.value), one(self.cost), one(self.quality))


class BudgetedAllocationEnv:
    """Single-episode view over a one-episode ``VectorEnv``."""

    def __init__(self, config: Optional[AllocationEnvConfig] = None):
        self.cfg = config or AllocationEnvConfig()
        self._v = VectorEnv(self.cfg, 1)
        self.history: List[StepInfo] = []

    @property
    def done(self) -> bool:
        return self._v.done

    @property
    def t(self) -> int:
        return self._v.t

    @property
    def remaining(self) -> float:
        return float(self._v.remaining[0])

    @property
    def pressure(self) -> float:
        return float(self._v.pressure[0])

    def reset(self, seed: Optional[int] = None) -> np.ndarray:
        self.history = []
        return self._v.reset([0 if seed is None else seed])[0]

    def step(self, action: int) -> Tuple[np.ndarray, float, bool, StepInfo]:
        obs, r, d, infos = self._v.step([int(action)])
        self.history.append(infos[0])
        return obs[0], float(r[0]), bool(d[0]), infos[0]

    def opportunity_stream(self) -> List[Opportunity]:
        v = self._v
        return [Opportunity(float(v.value[0, t]), float(v.cost[0, t]), float(v.quality[0, t]), float(v.season[0, t]))
                for t in range(self.cfg.horizon)]

    def state_dict(self) -> Dict[str, float]:
        v = self._v
        return {"t": v.t, "remaining": float(v.remaining[0]), "pressure": float(v.pressure[0]),
                "cum_spend": float(v.cum_spend[0]), "cum_value": float(v.cum_value[0])}
