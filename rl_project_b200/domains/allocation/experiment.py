"""Controlled offline experiments in the simulator: A/B tests and shadow evaluation.

A/B: episodes (identified by seed) go to the incumbent or challenger arm by
the same salted hash as serving traffic (``stable_bucket``), so assignment is
reproducible and policy-independent.  Per-episode metrics (value, spend,
pacing, violations, exhaustion, regret against the hindsight oracle) are
compared by difference of arm means with bootstrap intervals; the primary
metric (value) gets a two-sided permutation test.  Guardrails reject the
challenger when the value interval is unfavourable, utilisation leaves its
bounds, or violations / early exhaustion / listed metrics grow beyond their
allowed deltas.  ``ABResult.gate_metrics()`` flattens the result for
``PromotionGate`` (keys ``ab/<metric>_delta`` etc., as in
``src/forgeline/domains/allocation/experiment.py:97-118``).

Shadow: the incumbent acts; the candidate proposes an action at every step
from the same history without affecting it.  Reported: divergence rate, the
action confusion matrix, the candidate's OPE estimate on the incumbent's log
(when the incumbent is stochastic) and its simulator replay value on the
same seeds.
"""

from __future__ import annotations

import dataclasses
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.deployment.feature_flags import stable_bucket
from rl_project_b200.domains.allocation.env import AllocationEnvConfig, VectorEnv
from rl_project_b200.domains.allocation.ope import OPEConfig, OPEError, evaluate_target_policy
from rl_project_b200.domains.allocation.oracle import oracle_values
from rl_project_b200.domains.allocation.policies import Policy
from rl_project_b200.domains.allocation.rollout import aggregate_metrics, episode_metrics, run_episodes, seeds_for

PRIMARY = "value"
COMPARED = ("value", "spend", "utilization", "pacing_error", "violations", "early_exhaustion", "regret",
            "final_pressure")


@dataclass
class ABConfig:
    n_episodes: int = 400
    challenger_percent: float = 50.0
    salt: str = "forgeline-ab"
    seed: int = 0
    min_episodes: int = 30
    n_bootstrap: int = 1000
    n_permutations: int = 1000
    tolerance: float = 0.0
    utilization_bounds: Tuple[float, float] = (0.5, 1.0)
    max_violation_increase: float = 0.5
    max_exhaustion_increase: float = 0.1
    guardrails: Dict[str, float] = field(default_factory=dict)
    greedy: bool = False

    def validate(self) -> None:
        if self.n_episodes < 2 or not 0 < self.challenger_percent < 100 or self.min_episodes < 2:
            raise ConfigError("A/B needs n_episodes >= 2, 0 < challenger_percent < 100, min_episodes >= 2")
        if self.n_bootstrap < 10 or self.n_permutations < 10:
            raise ConfigError("n_bootstrap and n_permutations must be >= 10")


@dataclass
class ArmResult:
    name: str
    n: int
    metrics: Dict[str, float]
    per_episode: Dict[str, np.ndarray] = field(repr=False, default_factory=dict)


@dataclass
class MetricDelta:
    metric: str
    incumbent: float
    challenger: float
    delta: float
    ci_low: float
    ci_high: float
    std_error: float


@dataclass
class ABResult:
    incumbent: ArmResult
    challenger: ArmResult
    deltas: Dict[str, MetricDelta]
    p_value: float
    guardrail_failures: List[str]
    warnings: List[str]
    promote: bool
    elapsed_s: float

    def gate_metrics(self) -> Dict[str, float]:
        out: Dict[str, float] = {"ab/n_incumbent": float(self.incumbent.n), "ab/n_challenger": float(self.challenger.n),
                                 "ab/p_value": self.p_value, "ab/promote": float(self.promote)}
        for k, d in self.deltas.items():
            out.update({f"ab/{k}_delta": d.delta, f"ab/{k}_delta_ci_low": d.ci_low, f"ab/{k}_delta_ci_high": d.ci_high,
                        f"ab/{k}_challenger": d.challenger, f"ab/{k}_incumbent": d.incumbent})
        return out

    def to_dict(self) -> Dict[str, Any]:
        arm = lambda a: {"name": a.name, "n": a.n, "metrics": a.metrics}  # noqa: E731
        return {"incumbent": arm(self.incumbent), "challenger": arm(self.challenger),
                "deltas": {k: dataclasses.asdict(v) for k, v in self.deltas.items()}, "p_value": self.p_value,
                "guardrail_failures": self.guardrail_failures, "warnings": self.warnings, "promote": self.promote,
                "elapsed_s": self.elapsed_s}


def assign_arms(seeds: Sequence[int], challenger_percent: float, salt: str) -> Dict[int, str]:
    return {int(s): "challenger" if stable_bucket(str(s), salt) < challenger_percent * 100 else "incumbent"
            for s in seeds}


def _arm(name: str, policy: Policy, env_cfg: AllocationEnvConfig, seeds: List[int], greedy: bool,
         rng_seed: int) -> ArmResult:
    eps = run_episodes(policy, env_cfg, seeds, greedy=greedy, rng_seed=rng_seed)
    rows = [episode_metrics(e, env_cfg) for e in eps]
    per = {k: np.array([r[k] for r in rows]) for k in rows[0]}
    per["regret"] = oracle_values(env_cfg, seeds) - per["value"]
    return ArmResult(name, len(eps), {k: float(v.mean()) for k, v in per.items()}, per)


def bootstrap_delta(a: np.ndarray, b: np.ndarray, n_boot: int, rng: np.random.Generator):
    """Percentile interval and standard error of mean(b) - mean(a), arms resampled independently."""
    ia = rng.integers(0, len(a), size=(n_boot, len(a)))
    ib = rng.integers(0, len(b), size=(n_boot, len(b)))
    stats = b[ib].mean(1) - a[ia].mean(1)
    return float(np.quantile(stats, 0.025)), float(np.quantile(stats, 0.975)), float(stats.std(ddof=1))


def permutation_test(a: np.ndarray, b: np.ndarray, n_permutations: int, rng: np.random.Generator) -> float:
    """Two-sided randomisation p-value of the difference in means (with the +1 correction)."""
    observed = abs(b.mean() - a.mean())
    pooled = np.concatenate([a, b])
    n_a = len(a)
    perms = np.argsort(rng.random((n_permutations, len(pooled))), axis=1)
    shuffled = pooled[perms]
    diffs = np.abs(shuffled[:, n_a:].mean(1) - shuffled[:, :n_a].mean(1))
    return float((np.sum(diffs >= observed - 1e-15) + 1) / (n_permutations + 1))


def run_ab_experiment(incumbent: Policy, challenger: Policy, env_cfg: AllocationEnvConfig,
                      config: Optional[ABConfig] = None, incumbent_name: str = "incumbent",
                      challenger_name: str = "challenger") -> ABResult:
    cfg = config or ABConfig()
    cfg.validate()
    t0 = time.time()
    seeds = seeds_for(cfg.seed, cfg.n_episodes)
    arms = assign_arms(seeds, cfg.challenger_percent, cfg.salt)
    inc_seeds = [s for s in seeds if arms[s] == "incumbent"]
    ch_seeds = [s for s in seeds if arms[s] == "challenger"]
    warnings: List[str] = []
    if min(len(inc_seeds), len(ch_seeds)) < cfg.min_episodes:
        warnings.append(f"an arm has fewer than {cfg.min_episodes} episodes "
                        f"({len(inc_seeds)} incumbent / {len(ch_seeds)} challenger)")
    if not inc_seeds or not ch_seeds:
        raise ConfigError("both arms need at least one episode")
    inc = _arm(incumbent_name, incumbent, env_cfg, inc_seeds, cfg.greedy, cfg.seed + 1)
    ch = _arm(challenger_name, challenger, env_cfg, ch_seeds, cfg.greedy, cfg.seed + 2)
    rng = np.random.default_rng(cfg.seed)
    deltas = {}
    for k in COMPARED:
        lo, hi, se = bootstrap_delta(inc.per_episode[k], ch.per_episode[k], cfg.n_bootstrap, rng)
        deltas[k] = MetricDelta(k, inc.metrics[k], ch.metrics[k], ch.metrics[k] - inc.metrics[k], lo, hi, se)
    p = permutation_test(inc.per_episode[PRIMARY], ch.per_episode[PRIMARY], cfg.n_permutations, rng)
    fails: List[str] = []
    if deltas[PRIMARY].ci_low < -cfg.tolerance:
        fails.append(f"value delta CI lower bound {deltas[PRIMARY].ci_low:.4f} < -{cfg.tolerance}")
    lo_u, hi_u = cfg.utilization_bounds
    if not lo_u <= ch.metrics["utilization"] <= hi_u:
        fails.append(f"challenger utilization {ch.metrics['utilization']:.3f} outside [{lo_u}, {hi_u}]")
    if deltas["violations"].delta > cfg.max_violation_increase:
        fails.append(f"violations increased by {deltas['violations'].delta:.3f}")
    if deltas["early_exhaustion"].delta > cfg.max_exhaustion_increase:
        fails.append(f"early exhaustion increased by {deltas['early_exhaustion'].delta:.3f}")
    for metric, allowed in cfg.guardrails.items():
        if metric in ch.metrics and ch.metrics[metric] - inc.metrics.get(metric, 0.0) > allowed:
            fails.append(f"guardrail {metric} increased beyond {allowed}")
    return ABResult(inc, ch, deltas, p, fails, warnings, not fails and not warnings, time.time() - t0)


@dataclass
class ShadowResult:
    n_episodes: int
    divergence_rate: float
    confusion: List[List[int]]
    incumbent_value: float
    candidate_replay_value: float
    candidate_ope_value: Optional[float]
    ope_warnings: List[str]

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


def shadow_evaluate(incumbent: Policy, candidate: Policy, env_cfg: AllocationEnvConfig, seeds: Sequence[int],
                    ope_config: Optional[OPEConfig] = None, rng_seed: int = 0) -> ShadowResult:
    rng = np.random.default_rng(rng_seed)
    seeds = [int(s) for s in seeds]
    venv = VectorEnv(env_cfg, len(seeds))
    obs = venv.reset(seeds)
    incumbent.start(len(seeds))
    candidate.start(len(seeds))
    A = env_cfg.n_actions
    confusion = np.zeros((A, A), dtype=np.int64)
    while not venv.done:
        ctx = venv.context()
        a_inc, _ = incumbent.act(obs, ctx, rng, greedy=False)
        a_cand, _ = candidate.act(obs, ctx, rng, greedy=True)
        np.add.at(confusion, (np.asarray(a_inc, dtype=np.int64), np.asarray(a_cand, dtype=np.int64)), 1)
        obs, rewards, _, infos = venv.step(a_inc)
        spends = np.array([i.spend for i in infos])
        remaining = np.array([i.remaining_after for i in infos])
        incumbent.observe(a_inc, rewards, spends, remaining)
        candidate.observe(a_inc, rewards, spends, remaining)  # the shadow sees the served history
    inc_value = float(venv.cum_value.mean())
    replay = aggregate_metrics(run_episodes(candidate, env_cfg, seeds, greedy=True, rng_seed=rng_seed), env_cfg)
    ope_value, ope_warn = None, []
    if incumbent.stochastic:
        log = run_episodes(incumbent, env_cfg, seeds, rng_seed=rng_seed + 1)
        try:
            rep = evaluate_target_policy(candidate, log, env_cfg, ope_config or OPEConfig(n_bootstrap=200))
            ope_value = rep.estimates["dr"].value
            ope_warn = rep.diagnostics.warnings
        except OPEError as exc:
            ope_warn = [str(exc)]
    else:
        ope_warn = ["incumbent is deterministic: no propensities for off-policy evaluation"]
    total = int(confusion.sum())
    return ShadowResult(len(seeds), float(1.0 - np.trace(confusion) / max(total, 1)), confusion.tolist(), inc_value,
                        float(replay["value"]), ope_value, ope_warn)
