"""Off-policy evaluation of allocation policies from logged episodes.

With behaviour propensities b_t, target probabilities e_t of the logged
actions, per-decision ratios rho_t = e_t / b_t and cumulative weights
w_t = prod_{k<=t} rho_k (optionally clipped at ``max_weight``):

* IPS   (trajectory importance sampling)  mean_i w_{i,T-1} G_i
* SNIPS (self-normalised)                 sum_i w_{i,T-1} G_i / sum_i w_{i,T-1}
* PDIS  (per-decision)                    mean_i sum_t g^t w_{i,t} r_{i,t}
* DR    (per-decision doubly robust, Jiang & Li, ICML 2016)
        mean_i sum_t g^t [w_{i,t} (r_{i,t} - Q(h,a_t)) + w_{i,t-1} V(h)],  V(h) = sum_a e(a|h) Q(h,a)

with Q a ridge regression of the logged reward-to-go on [obs, onehot(a)].
Diagnostics: effective sample size (sum w)^2 / sum w^2, weight extremes,
support violations (target mass on actions the behaviour could not take --
refused beyond ``max_unsupported``), overlap sum_a min(e, b), and warnings on
weak support.  Percentile bootstrap intervals over episodes.  The report
layout (``estimates`` / ``diagnostics`` / ``logged_value``) matches
``src/forgeline/domains/allocation/ope.py:52-104``.  All estimators run on
``[n_episodes, T]`` arrays.
"""

from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence

import numpy as np

from rl_project_b200.core.errors import ForgelineError
from rl_project_b200.domains.allocation.env import AllocationEnvConfig, StepArrays
from rl_project_b200.domains.allocation.policies import Policy
from rl_project_b200.domains.allocation.rollout import Episode


class OPEError(ForgelineError):
    hint = "Check logged propensities and target-policy support; see the diagnostics in the message."


@dataclass
class OPEConfig:
    gamma: float = 1.0
    max_weight: Optional[float] = None
    min_ess: float = 10.0
    min_ess_fraction: float = 0.05
    max_unsupported: float = 0.0
    n_bootstrap: int = 500
    bootstrap_seed: int = 0
    ridge: float = 1e-2


@dataclass
class OPEEstimate:
    estimator: str
    value: float
    ci_low: float
    ci_high: float
    std_error: float


@dataclass
class OPEDiagnostics:
    n_episodes: int
    n_decisions: int
    ess: float
    ess_fraction: float
    max_weight: float
    mean_weight: float
    unsupported_fraction: float
    zero_target_fraction: float
    clipped_fraction: float
    overlap_mean: float
    overlap_min: float
    warnings: List[str] = field(default_factory=list)


@dataclass
class OPEReport:
    estimates: Dict[str, OPEEstimate]
    diagnostics: OPEDiagnostics
    logged_value: float
    target_name: str

    def to_dict(self) -> Dict[str, Any]:
        return {"target": self.target_name, "logged_value": self.logged_value,
                "estimates": {k: dataclasses.asdict(v) for k, v in self.estimates.items()},
                "diagnostics": dataclasses.asdict(self.diagnostics)}


def _stack(episodes: Sequence[Episode], A: int):
    T = len(episodes[0].steps)
    if any(len(e.steps) != T for e in episodes):
        raise OPEError("all logged episodes must have the same horizon")
    obs = np.array([[s.obs for s in e.steps] for e in episodes], dtype=np.float64)  # [n, T, 14]
    act = np.array([[s.action for s in e.steps] for e in episodes], dtype=np.int64)
    b = np.array([[s.propensity for s in e.steps] for e in episodes], dtype=np.float64)
    bp = np.array([[s.action_probs for s in e.steps] for e in episodes], dtype=np.float64)  # [n, T, A]
    r = np.array([[s.reward for s in e.steps] for e in episodes], dtype=np.float64)
    spend = np.array([[s.cost for s in e.steps] for e in episodes], dtype=np.float64)
    rem = np.array([[s.remaining_budget for s in e.steps] for e in episodes], dtype=np.float64)
    if bp.shape[2] != A:
        raise OPEError(f"logged action distributions have {bp.shape[2]} actions, the environment has {A}")
    return obs, act, b, bp, r, spend, rem


def target_probabilities(policy: Policy, episodes: Sequence[Episode], env_cfg: AllocationEnvConfig) -> List[np.ndarray]:
    """Replay all logged episodes through ``policy`` in lockstep, feeding it the logged actions and outcomes
    so stateful policies see the behaviour history; returns one ``[T, A]`` matrix per episode."""
    obs, act, _, _, r, spend, rem = _stack(episodes, env_cfg.n_actions)
    n, T = act.shape
    B = env_cfg.budget
    policy.start(n)
    out = np.zeros((n, T, env_cfg.n_actions))
    for t in range(T):
        o = obs[:, t]
        remaining = o[:, 0] * B
        ctx = StepArrays(t=t, horizon=env_cfg.horizon, remaining=remaining, budget=B, cum_spend=B - remaining,
                         value=(o[:, 3] + 1.0) * env_cfg.value_mean, cost=(o[:, 4] + 1.0) * env_cfg.cost_mean,
                         quality=o[:, 5])
        if hasattr(policy, "hist") and getattr(policy, "is_sequence", False):
            if policy.hist is None:
                policy.start(n)
            policy.hist.set_obs(o.astype(np.float32))
        out[:, t] = policy.action_probs(o.astype(np.float32), ctx)
        policy.observe(act[:, t], r[:, t], spend[:, t], rem[:, t])
    return [out[i] for i in range(n)]


def cumulative_weights(ratios: np.ndarray, max_weight: Optional[float] = None) -> np.ndarray:
    """Running products of the ratios along the last axis, optionally clipped at every step."""
    w = np.cumprod(ratios, axis=-1)
    if max_weight is not None:
        w = np.minimum(w, max_weight)
    return w


def ips_estimate(weights_final: np.ndarray, returns: np.ndarray) -> float:
    return float(np.mean(weights_final * returns))


def snips_estimate(weights_final: np.ndarray, returns: np.ndarray) -> float:
    s = float(np.sum(weights_final))
    return float(np.sum(weights_final * returns) / s) if s > 0 else float("nan")


def pdis_estimate(weights: np.ndarray, rewards: np.ndarray, gamma: float) -> float:
    disc = gamma ** np.arange(rewards.shape[-1])
    return float(np.mean((disc * weights * rewards).sum(-1)))


def dr_per_episode(weights: np.ndarray, rewards: np.ndarray, q_taken: np.ndarray, v_target: np.ndarray,
                   gamma: float) -> np.ndarray:
    disc = gamma ** np.arange(rewards.shape[-1])
    w_prev = np.concatenate([np.ones_like(weights[:, :1]), weights[:, :-1]], axis=1)
    return (disc * (weights * (rewards - q_taken) + w_prev * v_target)).sum(-1)


def dr_estimate(weights, rewards, q_taken, v_target, gamma: float) -> float:
    return float(np.mean(dr_per_episode(np.asarray(weights), np.asarray(rewards), np.asarray(q_taken),
                                        np.asarray(v_target), gamma)))


def effective_sample_size(weights_final: np.ndarray) -> float:
    s2 = float(np.sum(weights_final ** 2))
    return float(np.sum(weights_final)) ** 2 / s2 if s2 > 0 else 0.0


def bootstrap_ci(per_episode: np.ndarray, n_bootstrap: int, seed: int, level: float = 0.95,
                 stat: Callable[[np.ndarray], float] = np.mean):
    """Percentile interval and standard error of ``stat`` over episode resamples."""
    x = np.asarray(per_episode, dtype=np.float64)
    if n_bootstrap < 2 or len(x) < 2:
        v = float(stat(x))
        return v, v, 0.0
    rng = np.random.default_rng(seed)
    idx = rng.integers(0, len(x), size=(n_bootstrap, len(x)))
    boots = np.array([stat(x[i]) for i in idx]) if stat is not np.mean else x[idx].mean(1)
    a = (1.0 - level) / 2.0
    return float(np.quantile(boots, a)), float(np.quantile(boots, 1.0 - a)), float(boots.std(ddof=1))


def _features(obs: np.ndarray, actions: np.ndarray, A: int) -> np.ndarray:
    onehot = np.eye(A)[actions]
    return np.concatenate([obs, onehot, np.ones(obs.shape[:-1] + (1,))], axis=-1)


def fit_q_ridge(obs: np.ndarray, actions: np.ndarray, rewards: np.ndarray, A: int, gamma: float,
                ridge: float) -> np.ndarray:
    """Ridge regression of the logged reward-to-go on [obs, onehot(a), 1]."""
    T = rewards.shape[1]
    disc = gamma ** np.arange(T)
    togo = np.flip(np.cumsum(np.flip(rewards * disc, 1), 1), 1) / disc
    X = _features(obs, actions, A).reshape(-1, obs.shape[-1] + A + 1)
    y = togo.reshape(-1)
    return np.linalg.solve(X.T @ X + ridge * np.eye(X.shape[1]), X.T @ y)


def q_values(theta: np.ndarray, obs: np.ndarray, A: int) -> np.ndarray:
    """``Q(h, a)`` for every action: ``[..., A]``."""
    lead = obs.shape[:-1]
    feats = np.stack([_features(obs, np.full(lead, a, dtype=np.int64), A) for a in range(A)], -2)
    return feats @ theta


def evaluate_policy(episodes: Sequence[Episode], target_probs: Sequence[np.ndarray], env_cfg: AllocationEnvConfig,
                    config: Optional[OPEConfig] = None, target_name: str = "target") -> OPEReport:
    cfg = config or OPEConfig()
    if not episodes:
        raise OPEError("no logged episodes")
    if len(target_probs) != len(episodes):
        raise OPEError("one target probability matrix per episode is required")
    A = env_cfg.n_actions
    obs, act, b, bp, r, _, _ = _stack(episodes, A)
    n, T = act.shape
    tp = np.stack([np.asarray(x, dtype=np.float64) for x in target_probs])
    if tp.shape != (n, T, A):
        raise OPEError(f"target probabilities have shape {tp.shape}, expected {(n, T, A)}")
    if not np.isfinite(tp).all() or (tp < -1e-12).any() or (np.abs(tp.sum(-1) - 1.0) > 1e-6).any():
        raise OPEError("target probabilities are not valid distributions")
    if not np.isfinite(b).all() or (b <= 0).any():
        raise OPEError("logged behaviour propensities must be positive and finite")
    e = np.take_along_axis(tp, act[..., None], -1)[..., 0]
    unsupported = int(((bp <= 0) & (tp > 0)).any(-1).sum())
    n_dec = n * T
    if unsupported / n_dec > cfg.max_unsupported:
        raise OPEError(f"target policy is unsupported by the log at {unsupported}/{n_dec} decisions "
                       f"(tolerance {cfg.max_unsupported:.2%})")
    ratios = e / b
    w = cumulative_weights(ratios)
    wf = w[:, -1]
    if not np.isfinite(wf).all():
        raise OPEError("importance weights overflowed to non-finite values")
    disc = cfg.gamma ** np.arange(T)
    returns = (disc * r).sum(1)
    overlap = np.minimum(tp, bp).sum(-1)
    ess = effective_sample_size(wf)
    zero_frac = float((e <= 0).sum()) / n_dec
    diag = OPEDiagnostics(n, n_dec, ess, ess / n, float(wf.max()), float(wf.mean()), unsupported / n_dec, zero_frac,
                          0.0, float(overlap.mean()), float(overlap.min()))
    if zero_frac > 0.5:
        diag.warnings.append(f"target gives zero probability to {zero_frac:.0%} of logged actions")
    if ess < cfg.min_ess:
        diag.warnings.append(f"effective sample size {ess:.1f} < {cfg.min_ess}: estimates unreliable")
    if ess / n < cfg.min_ess_fraction:
        diag.warnings.append(f"ESS fraction {ess / n:.3f} < {cfg.min_ess_fraction}: weak overlap")
    if diag.max_weight > 100.0:
        diag.warnings.append(f"maximum trajectory weight {diag.max_weight:.1f} dominates the estimate")

    est: Dict[str, OPEEstimate] = {}

    def add(name: str, per_episode: np.ndarray, value: float, stat=np.mean) -> None:
        if not math.isfinite(value):
            raise OPEError(f"{name} estimate is non-finite")
        lo, hi, se = bootstrap_ci(per_episode, cfg.n_bootstrap, cfg.bootstrap_seed, stat=stat)
        est[name] = OPEEstimate(name, value, lo, hi, se)

    theta = fit_q_ridge(obs, act, r, A, cfg.gamma, cfg.ridge)
    qs = q_values(theta, obs, A)  # [n, T, A]
    q_taken = np.take_along_axis(qs, act[..., None], -1)[..., 0]
    v_tgt = (tp * qs).sum(-1)

    def family(weights: np.ndarray, suffix: str) -> None:
        final = weights[:, -1]
        add("ips" + suffix, final * returns, ips_estimate(final, returns))
        pd = (disc * weights * r).sum(1)
        add("pdis" + suffix, pd, float(pd.mean()))
        dr = dr_per_episode(weights, r, q_taken, v_tgt, cfg.gamma)
        add("dr" + suffix, dr, float(dr.mean()))

    family(w, "")
    if wf.sum() > 0:
        pairs = np.stack([wf, returns], 1)
        add("snips", pairs, snips_estimate(wf, returns), stat=lambda x: snips_estimate(x[:, 0], x[:, 1])
            if x[:, 0].sum() > 0 else snips_estimate(wf, returns))
    else:
        diag.warnings.append("SNIPS unavailable: every trajectory weight is zero")
    if cfg.max_weight is not None:
        wc = cumulative_weights(ratios, cfg.max_weight)
        diag.clipped_fraction = float((np.abs(wc - w) > 1e-12).any(1).mean())
        family(wc, "_clipped")
    return OPEReport(est, diag, float(returns.mean()), target_name)


def evaluate_target_policy(policy: Policy, episodes: Sequence[Episode], env_cfg: AllocationEnvConfig,
                           config: Optional[OPEConfig] = None, target_name: Optional[str] = None) -> OPEReport:
    tp = target_probabilities(policy, episodes, env_cfg)
    return evaluate_policy(episodes, tp, env_cfg, config, target_name or policy.name)
