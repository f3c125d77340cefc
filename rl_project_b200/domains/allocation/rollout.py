"""Logged allocation episodes: the JSONL log format, the batched episode runner and
budget / pacing metrics.

The log format (one ``LoggedStep`` per line with ``schema_version`` 1) and the
metric keys follow ``src/forgeline/domains/allocation/rollout.py:19-208`` so
logs and reports move between the two frameworks.  Behaviour propensities and
full action distributions are logged for off-policy evaluation.
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
import math
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, Iterable, List, Sequence

import numpy as np

from rl_project_b200.core.errors import DatasetError
from rl_project_b200.domains.allocation.env import AllocationEnvConfig, VectorEnv
from rl_project_b200.domains.allocation.policies import Policy

SCHEMA_VERSION = 1


@dataclass
class LoggedStep:
    episode_id: str
    seed: int
    t: int
    obs: List[float]
    history_summary: Dict[str, float]
    action: int
    propensity: float
    action_probs: List[float]
    reward: float
    cost: float
    next_obs: List[float]
    cum_spend: float
    cum_reward: float
    remaining_budget: float
    terminal: bool
    clipped: bool
    pressure: float  # latent state: logged for analysis, never shown to policies

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


@dataclass
class Episode:
    episode_id: str
    seed: int
    steps: List[LoggedStep]

    @property
    def total_reward(self) -> float:
        return float(sum(s.reward for s in self.steps))

    @property
    def total_spend(self) -> float:
        return float(sum(s.cost for s in self.steps))


def write_episodes(episodes: Iterable[Episode], path: str | Path) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("w") as fh:
        for ep in episodes:
            for s in ep.steps:
                fh.write(json.dumps({**s.to_dict(), "schema_version": SCHEMA_VERSION}) + "\n")
    return path


def validate_step(step: LoggedStep, where: str = "") -> None:
    p = step.propensity
    if not (isinstance(p, (int, float)) and math.isfinite(p) and 0.0 < p <= 1.0 + 1e-9):
        raise DatasetError(f"{where}: propensity {p!r} is not in (0, 1]")
    probs = np.asarray(step.action_probs, dtype=float)
    if probs.ndim != 1 or not np.isfinite(probs).all() or (probs < 0).any() or abs(probs.sum() - 1.0) > 1e-6:
        raise DatasetError(f"{where}: action_probs must be a finite probability vector")
    if not 0 <= step.action < len(probs) or abs(probs[step.action] - p) > 1e-6:
        raise DatasetError(f"{where}: propensity {p} does not match action_probs[{step.action}]")
    if not (math.isfinite(step.reward) and math.isfinite(step.cost)) or step.cost < -1e-12:
        raise DatasetError(f"{where}: non-finite reward/cost or negative cost")


def read_episodes(path: str | Path) -> List[Episode]:
    """Read and validate a log written by ``write_episodes`` (schema, propensities, complete episodes)."""
    episodes: Dict[str, Episode] = {}
    for n, line in enumerate(Path(path).read_text().splitlines(), 1):
        if not line.strip():
            continue
        try:
            d = json.loads(line)
        except json.JSONDecodeError as exc:
            raise DatasetError(f"{path}:{n}: invalid JSON ({exc})") from None
        if d.pop("schema_version", None) != SCHEMA_VERSION:
            raise DatasetError(f"{path}:{n}: unsupported schema_version")
        try:
            step = LoggedStep(**d)
        except TypeError as exc:
            raise DatasetError(f"{path}:{n}: malformed logged step ({exc})") from None
        validate_step(step, f"{path}:{n}")
        episodes.setdefault(step.episode_id, Episode(step.episode_id, step.seed, [])).steps.append(step)
    for ep in episodes.values():
        ep.steps.sort(key=lambda s: s.t)
        if [s.t for s in ep.steps] != list(range(len(ep.steps))):
            raise DatasetError(f"episode {ep.episode_id} has missing or duplicate timesteps")
        if not ep.steps[-1].terminal:
            raise DatasetError(f"episode {ep.episode_id} is not terminated")
    return list(episodes.values())


def episode_seed(base_seed: int, index: int) -> int:
    """Independent 31-bit episode seeds derived by hashing (base, index)."""
    h = hashlib.blake2b(f"{base_seed}/{index}".encode(), digest_size=8).digest()
    return int.from_bytes(h, "little") % (2 ** 31 - 1)


def seeds_for(base_seed: int, n_episodes: int, offset: int = 0) -> List[int]:
    return [episode_seed(base_seed, offset + i) for i in range(n_episodes)]


def run_episodes(policy: Policy, env_cfg: AllocationEnvConfig, seeds: Sequence[int], *, greedy: bool = False,
                 rng_seed: int = 0, episode_prefix: str = "", batch: int = 256) -> List[Episode]:
    """One fully logged episode per seed, stepped in lockstep batches."""
    rng = np.random.default_rng(rng_seed)
    out: List[Episode] = []
    seeds = [int(s) for s in seeds]
    B = env_cfg.budget
    for lo in range(0, len(seeds), batch):
        chunk = seeds[lo:lo + batch]
        venv = VectorEnv(env_cfg, len(chunk))
        obs = venv.reset(chunk)
        policy.start(len(chunk))
        logs: List[List[LoggedStep]] = [[] for _ in chunk]
        while not venv.done:
            actions, probs = policy.act(obs, venv.context(), rng, greedy=greedy)
            actions = np.asarray(actions, dtype=np.int64)
            next_obs, rewards, dones, infos = venv.step(actions)
            for j, info in enumerate(infos):
                logs[j].append(LoggedStep(
                    episode_id=f"{episode_prefix}{chunk[j]}", seed=chunk[j], t=info.t, obs=obs[j].tolist(),
                    history_summary={"cum_spend_frac": (B - info.remaining_before) / B,
                                     "elapsed_frac": info.t / env_cfg.horizon},
                    action=int(actions[j]), propensity=float(probs[j, actions[j]]),
                    action_probs=[float(x) for x in probs[j]], reward=info.reward, cost=info.spend,
                    next_obs=next_obs[j].tolist(), cum_spend=float(venv.cum_spend[j]),
                    cum_reward=float(venv.cum_value[j]), remaining_budget=info.remaining_after,
                    terminal=bool(dones[j]), clipped=info.clipped, pressure=info.pressure_after))
            policy.observe(actions, rewards, np.array([i.spend for i in infos]),
                           np.array([i.remaining_after for i in infos]))
            obs = next_obs
        out.extend(Episode(f"{episode_prefix}{s}", s, logs[j]) for j, s in enumerate(chunk))
    return out


def episode_metrics(ep: Episode, env_cfg: AllocationEnvConfig, exhaustion_frac: float = 0.9) -> Dict[str, float]:
    T, B = env_cfg.horizon, env_cfg.budget
    spend = np.array([s.cost for s in ep.steps])
    reward = np.array([s.reward for s in ep.steps])
    frac = np.cumsum(spend) / B
    gap = np.abs(frac - np.arange(1, T + 1) / T)
    hit = np.nonzero(frac >= 1.0 - 1e-9)[0]
    exhausted = bool(hit.size and hit[0] < exhaustion_frac * T - 1)
    parts = np.array_split(np.arange(T), 3)
    counts = np.bincount([s.action for s in ep.steps], minlength=env_cfg.n_actions) / T
    m = {"value": reward.sum(), "spend": spend.sum(), "utilization": spend.sum() / B,
         "value_per_budget": reward.sum() / B, "pacing_error": gap.mean(), "early_exhaustion": float(exhausted),
         "unused_budget_frac": max(0.0, 1.0 - spend.sum() / B), "violations": float(sum(s.clipped for s in ep.steps)),
         "reward_variance": reward.var(), "final_pressure": ep.steps[-1].pressure}
    for name, idx in zip(("early", "mid", "late"), parts):
        m[f"value_{name}"] = reward[idx].sum()
        m[f"spend_{name}"] = spend[idx].sum()
    m.update({f"action_frac_{i}": counts[i] for i in range(env_cfg.n_actions)})
    return {k: float(v) for k, v in m.items()}


def aggregate_metrics(episodes: Sequence[Episode], env_cfg: AllocationEnvConfig) -> Dict[str, float]:
    rows = [episode_metrics(e, env_cfg) for e in episodes]
    out: Dict[str, float] = {"n_episodes": float(len(rows))}
    for k in rows[0]:
        v = np.array([r[k] for r in rows])
        out[k] = float(v.mean())
        out[f"{k}_std"] = float(v.std(ddof=1)) if len(v) > 1 else 0.0
    out["value_ci95_halfwidth"] = 1.96 * out["value_std"] / math.sqrt(len(rows)) if len(rows) > 1 else 0.0
    return out
