"""End-to-end allocation benchmark: baselines vs PPO policies, OPE, A/B and shadow.

Policies: the threshold heuristic, the dual pacer, and PPO with an MLP and a
GRU actor-critic trained by the framework ``Trainer`` for every training seed.
Each is evaluated on a held-out seed family with regret against the hindsight
oracle.  The best PPO policy is then judged offline (OPE on an epsilon-mixed
dual-pacer log), in a simulated A/B test against the dual pacer, and in a
shadow run.  Writes ``results.json`` and ``summary.md`` under ``output_dir``.
Config keys follow ``src/forgeline/domains/allocation/benchmark.py:37-57``.
"""

from __future__ import annotations

import dataclasses
import json
import platform
import time
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Dict, List, Optional

import numpy as np
import torch

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.domains.allocation.env import ACTION_NAMES, AllocationEnvConfig, strict_config
from rl_project_b200.domains.allocation.experiment import ABConfig, run_ab_experiment, shadow_evaluate
from rl_project_b200.domains.allocation.ope import OPEConfig, OPEError, evaluate_target_policy
from rl_project_b200.domains.allocation.oracle import oracle_values
from rl_project_b200.domains.allocation.policies import (DualPacingPolicy, EpsilonMixPolicy, Policy, PolicyNetConfig,
                                                         ThresholdPacingPolicy)
from rl_project_b200.domains.allocation.ppo import AllocationPPOAlgorithm, AllocationPPOConfig
from rl_project_b200.domains.allocation.rollout import aggregate_metrics, run_episodes, seeds_for


@dataclass
class BenchmarkConfig:
    env: Dict[str, Any] = field(default_factory=dict)
    training_seeds: List[int] = field(default_factory=lambda: [0, 1, 2, 3, 4])
    eval_episodes: int = 300
    eval_seed: int = 20_000
    trainer_steps: int = 600
    episodes_per_rollout: int = 32
    ppo_epochs: int = 4
    learning_rate: float = 3e-3
    hidden: int = 64
    window: int = 8
    heuristic_threshold: float = 0.6
    dual_learning_rate: float = 0.2
    dual_initial_price: float = 0.8
    ope_log_episodes: int = 300
    ope_epsilon: float = 0.2
    ope_max_weight: Optional[float] = 20.0
    ab_episodes: int = 400
    shadow_episodes: int = 100
    output_dir: str = "runs/allocation-benchmark"
    metrics: str = "local"
    policies: List[str] = field(default_factory=lambda: ["mlp", "gru"])

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "BenchmarkConfig":
        return strict_config(cls, d, "benchmark")


def train_policy(kind: str, env_cfg: AllocationEnvConfig, bcfg: BenchmarkConfig, seed: int, out_dir: Path,
                 metrics: str):
    """Train one PPO policy through the standard Trainer; returns (policy, seconds, checkpoint dir)."""
    from rl_project_b200.core.config import (CheckpointConfig, ExperimentManifest, OptimizerConfig, ScheduleConfig,
                                             TrainerConfig)
    from rl_project_b200.core.lifecycle import RunContext
    from rl_project_b200.training.common.trainer import Trainer

    net_cfg = PolicyNetConfig(kind=kind, hidden=bcfg.hidden, window=bcfg.window)
    ppo_cfg = AllocationPPOConfig(episodes_per_rollout=bcfg.episodes_per_rollout, ppo_epochs=bcfg.ppo_epochs, seed=seed)
    manifest = ExperimentManifest(
        name=f"allocation-ppo-{kind}-seed{seed}", algorithm="allocation_ppo", output_dir=str(out_dir),
        trainer=TrainerConfig(max_steps=bcfg.trainer_steps, batch_size=1, gradient_accumulation_steps=4, eval_every=0,
                              log_every=50, device="cpu", seed=seed,
                              optimizer=OptimizerConfig(learning_rate=bcfg.learning_rate, weight_decay=0.0, beta2=0.999,
                                                        grad_clip=0.5, decay_only_matrices=False),
                              schedule=ScheduleConfig(name="linear_decay", warmup_steps=0,
                                                      decay_steps=bcfg.trainer_steps, min_lr=bcfg.learning_rate / 10),
                              checkpoint=CheckpointConfig(directory="checkpoints", save_every=0)),
        algorithm_params={"env": env_cfg.to_dict(), "policy": net_cfg.to_dict(),
                          "episodes_per_rollout": bcfg.episodes_per_rollout, "ppo_epochs": bcfg.ppo_epochs,
                          "seed": seed})
    ctx = RunContext.create(manifest, metrics_backend=metrics)
    torch.manual_seed(seed)
    alg = AllocationPPOAlgorithm(env_cfg, net_cfg, ppo_cfg)
    t0 = time.time()
    Trainer(ctx, alg).fit()
    ctx.close()
    return alg.policy, time.time() - t0, str(Path(ctx.output_dir) / "checkpoints" / "final")


def evaluate(policy: Policy, env_cfg: AllocationEnvConfig, seeds: List[int], oracle: np.ndarray) -> Dict[str, float]:
    t0 = time.time()
    eps = run_episodes(policy, env_cfg, seeds, rng_seed=seeds[0])
    m = aggregate_metrics(eps, env_cfg)
    regret = oracle - np.array([e.total_reward for e in eps])
    m["regret_vs_oracle"] = float(regret.mean())
    m["regret_vs_oracle_std"] = float(regret.std(ddof=1)) if len(regret) > 1 else 0.0
    m["eval_seconds"] = time.time() - t0
    m["env_steps_per_sec"] = len(seeds) * env_cfg.horizon / max(m["eval_seconds"], 1e-9)
    return m


def run_benchmark(bcfg: BenchmarkConfig, log: Callable[[str], None] = print) -> Dict[str, Any]:
    env_cfg = AllocationEnvConfig.from_dict(bcfg.env)
    out = Path(bcfg.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    seeds = seeds_for(bcfg.eval_seed, bcfg.eval_episodes)
    oracle = oracle_values(env_cfg, seeds)
    res: Dict[str, Any] = {"config": dataclasses.asdict(bcfg), "env": env_cfg.to_dict(),
                           "action_names": list(ACTION_NAMES),
                           "oracle": {"mean_value": float(oracle.mean()),
                                      "std": float(oracle.std(ddof=1)) if len(oracle) > 1 else 0.0},
                           "environment": {"python": platform.python_version(), "torch": torch.__version__,
                                           "platform": platform.platform()},
                           "policies": {}}
    heuristic = ThresholdPacingPolicy(env_cfg, threshold=bcfg.heuristic_threshold)
    dual = DualPacingPolicy(env_cfg, learning_rate=bcfg.dual_learning_rate, initial_price=bcfg.dual_initial_price)
    for name, pol in (("heuristic", heuristic), ("dual_pacing", dual)):
        res["policies"][name] = {"eval": evaluate(pol, env_cfg, seeds, oracle)}
        log(f"{name}: value {res['policies'][name]['eval']['value']:.3f}")
    best_policy, best_value, best_name = None, -np.inf, ""
    for kind in bcfg.policies:
        runs = []
        for seed in bcfg.training_seeds:
            pol, secs, ckpt = train_policy(kind, env_cfg, bcfg, seed, out / f"ppo_{kind}" / f"seed{seed}", bcfg.metrics)
            ev = evaluate(pol, env_cfg, seeds, oracle)
            runs.append({"seed": seed, "train_seconds": secs, "checkpoint": ckpt, "eval": ev})
            if ev["value"] > best_value:
                best_policy, best_value, best_name = pol, ev["value"], f"ppo_{kind}/seed{seed}"
            log(f"ppo_{kind} seed {seed}: value {ev['value']:.3f} ({secs:.0f}s)")
        vals = np.array([r["eval"]["value"] for r in runs])
        res["policies"][f"ppo_{kind}"] = {"runs": runs, "value_mean": float(vals.mean()),
                                          "value_std_across_seeds": float(vals.std(ddof=1)) if len(vals) > 1 else 0.0}
    if best_policy is not None:
        logged = run_episodes(EpsilonMixPolicy(dual, bcfg.ope_epsilon, env_cfg.n_actions), env_cfg,
                              seeds_for(bcfg.eval_seed + 1, bcfg.ope_log_episodes), rng_seed=1)
        try:
            rep = evaluate_target_policy(EpsilonMixPolicy(best_policy, bcfg.ope_epsilon, env_cfg.n_actions), logged,
                                         env_cfg, OPEConfig(max_weight=bcfg.ope_max_weight, n_bootstrap=200))
            res["ope"] = {"target": best_name, **rep.to_dict()}
        except OPEError as exc:
            res["ope"] = {"target": best_name, "error": str(exc)}
        ab = run_ab_experiment(dual, best_policy, env_cfg, ABConfig(n_episodes=bcfg.ab_episodes, seed=bcfg.eval_seed),
                               incumbent_name="dual_pacing", challenger_name=best_name)
        res["ab"] = ab.to_dict()
        res["shadow"] = shadow_evaluate(EpsilonMixPolicy(dual, bcfg.ope_epsilon, env_cfg.n_actions), best_policy,
                                        env_cfg, seeds_for(bcfg.eval_seed + 2, bcfg.shadow_episodes)).to_dict()
    (out / "results.json").write_text(json.dumps(res, indent=2, default=float))
    (out / "summary.md").write_text(render_summary(res))
    return res


def render_summary(r: Dict[str, Any]) -> str:
    lines = ["# Allocation benchmark", "", f"Hindsight oracle (no pressure): {r['oracle']['mean_value']:.3f}", "",
             "| policy | value | regret vs oracle | utilization | pacing error | violations |", "|---|---|---|---|---|---|"]
    for name, p in r["policies"].items():
        evs = [p["eval"]] if "eval" in p else [x["eval"] for x in p["runs"]]
        mean = lambda k: float(np.mean([e[k] for e in evs]))  # noqa: E731
        lines.append(f"| {name} | {mean('value'):.3f} | {mean('regret_vs_oracle'):.3f} | {mean('utilization'):.3f} | "
                     f"{mean('pacing_error'):.3f} | {mean('violations'):.2f} |")
    if "ope" in r and "estimates" in r["ope"]:
        lines += ["", f"OPE of {r['ope']['target']} (eps-mixed) on a dual-pacer log: " + ", ".join(
            f"{k} {v['value']:.3f}" for k, v in r["ope"]["estimates"].items()),
            f"ESS {r['ope']['diagnostics']['ess']:.1f}; warnings: {r['ope']['diagnostics']['warnings'] or 'none'}"]
    if "ab" in r:
        d = r["ab"]["deltas"]["value"]
        lines += ["", f"A/B (simulated) dual_pacing vs {r['ab']['challenger']['name']}: value delta {d['delta']:.3f} "
                      f"[{d['ci_low']:.3f}, {d['ci_high']:.3f}], p = {r['ab']['p_value']:.4f}, "
                      f"promote = {r['ab']['promote']}"]
    if "shadow" in r:
        s = r["shadow"]
        lines += ["", f"Shadow: divergence {s['divergence_rate']:.2%}, candidate replay value "
                      f"{s['candidate_replay_value']:.3f}"]
    return "\n".join(lines) + "\n"
