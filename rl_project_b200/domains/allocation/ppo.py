"""PPO for allocation policies, run by the framework's ``Trainer`` (algorithm ``allocation_ppo``).

Design: a rollout writes straight into a :class:`Trajectory`, a set of ``[T, n, ...]`` tensors on the
algorithm's device, so the network's outputs never leave the device during collection except for the
sampled actions the CPU environment needs.  Advantages are computed for all episodes and all steps at
once as one matrix product with the GAE discount operator (an upper-triangular ``[T, T]`` matrix of
``(gamma * lambda) ** (s - t)``), instead of a backward recursion.  A rollout is reused for
``ppo_epochs`` optimiser steps with a fresh permutation each step; micro-batches are strided slices of
that permutation.

Interfaces kept as the reference defines them (``src/forgeline/domains/allocation/ppo.py``): the
``AllocationPPOConfig`` field names and defaults, the algorithm name, ``build_allocation_ppo`` taking
``{env: {...}, policy: {...}, <config fields>}``, and the checkpoint ``model_spec``
``{family: allocation_policy, policy, env}`` that ``load_allocation_policy`` reads back
(``src/forgeline/domains/allocation/ppo.py:190-217``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Mapping, Optional

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.domains.allocation.env import OBS_DIM, AllocationEnvConfig, VectorEnv, strict_config
from rl_project_b200.domains.allocation.policies import (NeuralPolicy, PolicyNetConfig, build_actor_critic,
                                                         history_feature_dim)
from rl_project_b200.domains.allocation.rollout import aggregate_metrics, run_episodes, seeds_for
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm
from rl_project_b200.training.ppo import ppo_clipped_objective

_EVAL_KEYS = ("value", "value_std", "utilization", "pacing_error", "early_exhaustion", "violations",
              "final_pressure")


@dataclass
class AllocationPPOConfig:
    episodes_per_rollout: int = 16
    ppo_epochs: int = 4
    clip_ratio: float = 0.2
    value_coef: float = 0.5
    entropy_coef: float = 0.01
    gamma: float = 1.0
    gae_lambda: float = 0.95
    normalize_advantages: bool = True
    eval_episodes: int = 64
    eval_seed: int = 10_000
    seed: int = 0

    def validate(self) -> None:
        rules = (
            (min(self.episodes_per_rollout, self.ppo_epochs, self.eval_episodes) >= 1,
             "episodes_per_rollout, ppo_epochs and eval_episodes must be >= 1"),
            (0 < self.clip_ratio < 1 and 0 < self.gamma <= 1 and 0 <= self.gae_lambda <= 1,
             "clip_ratio in (0,1), gamma in (0,1], gae_lambda in [0,1] required"),
        )
        for ok, msg in rules:
            if not ok:
                raise ConfigError(msg)

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "AllocationPPOConfig":
        return strict_config(cls, d, "AllocationPPOConfig")


def gae_operator(T: int, gamma: float, lam: float, device=None, dtype=torch.float32) -> torch.Tensor:
    """``D[t, s] = (gamma * lam) ** (s - t)`` for ``s >= t`` (else 0): advantages = ``D @ deltas``."""
    steps = torch.arange(T, device=device, dtype=dtype)
    lag = steps[None, :] - steps[:, None]
    return torch.where(lag >= 0, (gamma * lam) ** lag.clamp(min=0), torch.zeros((), device=device, dtype=dtype))


def batched_gae(rewards, values, gamma: float, lam: float):
    """GAE over ``[T, n]`` rewards and ``[T+1, n]`` values (terminal value 0) for every episode at once:
    returns (advantages ``[T, n]``, returns ``[T, n]``).  Accepts numpy arrays or tensors."""
    as_np = isinstance(rewards, np.ndarray)
    r = torch.as_tensor(rewards, dtype=torch.float64)
    v = torch.as_tensor(values, dtype=torch.float64, device=r.device)
    deltas = r + gamma * v[1:] - v[:-1]
    adv = gae_operator(r.shape[0], gamma, lam, r.device, torch.float64) @ deltas
    ret = adv + v[:-1]
    if as_np:
        return adv.numpy().astype(rewards.dtype), ret.numpy().astype(rewards.dtype)
    return adv.to(rewards.dtype), ret.to(rewards.dtype)


@dataclass
class Trajectory:
    """One rollout of ``n`` episodes over ``T`` steps, stored step-major on the device."""

    obs: torch.Tensor                     # [T, n, OBS_DIM]
    actions: torch.Tensor                 # [T, n] int64
    logp: torch.Tensor                    # [T, n]
    values: torch.Tensor                  # [T + 1, n]; the last row stays 0 (terminal)
    rewards: torch.Tensor                 # [T, n]
    hist: Optional[torch.Tensor] = None   # [T, n, W, D] for sequence policies
    lengths: Optional[torch.Tensor] = None

    @classmethod
    def empty(cls, T: int, n: int, device, window: int = 0, hist_dim: int = 0) -> "Trajectory":
        z = lambda *s, dt=torch.float32: torch.zeros(*s, device=device, dtype=dt)  # noqa: E731
        seq = window > 0
        return cls(z(T, n, OBS_DIM), z(T, n, dt=torch.int64), z(T, n), z(T + 1, n), z(T, n),
                   z(T, n, window, hist_dim) if seq else None, z(T, n, dt=torch.int64) if seq else None)


@dataclass
class RolloutBatch:
    """Flattened ``[T * n]`` training view of a :class:`Trajectory` with its advantages."""

    obs: torch.Tensor
    hist: Optional[torch.Tensor]
    lengths: Optional[torch.Tensor]
    actions: torch.Tensor
    old_logp: torch.Tensor
    advantages: torch.Tensor
    returns: torch.Tensor
    perm: torch.Tensor
    stats: Dict[str, float] = field(default_factory=dict)

    def features(self, idx: torch.Tensor):
        return self.obs[idx] if self.hist is None else (self.obs[idx], self.hist[idx], self.lengths[idx])


class AllocationPPOAlgorithm(PostTrainingAlgorithm):
    name = "allocation_ppo"

    def __init__(self, env_cfg: AllocationEnvConfig, net_cfg: PolicyNetConfig, config: AllocationPPOConfig,
                 device: torch.device | str = "cpu"):
        for c in (env_cfg, net_cfg, config):
            c.validate()
        self.env_cfg, self.net_cfg, self.cfg = env_cfg, net_cfg, config
        self.device = torch.device(device)
        self.net = build_actor_critic(env_cfg.n_actions, net_cfg).to(self.device)
        self.policy = NeuralPolicy(self.net, env_cfg, self.device)
        self.rng = np.random.default_rng(config.seed)
        self._gae = gae_operator(env_cfg.horizon, config.gamma, config.gae_lambda, self.device)
        self._batch: Optional[RolloutBatch] = None
        self._episodes_seen = 0

    # ------------------------------------------------------------------ trainer protocol
    def parameters(self) -> List[nn.Parameter]:
        return [p for p in self.net.parameters() if p.requires_grad]

    def modules(self):
        return (self.net,)

    def collect(self, step: int) -> RolloutBatch:
        fresh = self._batch is None or step % self.cfg.ppo_epochs == 0
        if fresh:
            self._batch = self._to_batch(*self._roll())
        self._batch.perm = torch.as_tensor(self.rng.permutation(self._batch.actions.numel()), device=self.device)
        return self._batch

    def loss(self, batch: RolloutBatch, micro_step: int, n_micro: int):
        idx = batch.perm[micro_step::n_micro]
        logits, values = self.net(batch.features(idx))
        logp_all = F.log_softmax(logits, -1)
        logp = logp_all.gather(1, batch.actions[idx, None]).squeeze(1)
        log_ratio = logp - batch.old_logp[idx]
        ratio = log_ratio.exp()
        terms = {
            "policy_loss": ppo_clipped_objective(ratio, batch.advantages[idx], self.cfg.clip_ratio).mean(),
            "value_loss": F.mse_loss(values, batch.returns[idx]),
            "entropy": -(logp_all.exp() * logp_all).sum(-1).mean(),
        }
        loss = terms["policy_loss"] + self.cfg.value_coef * terms["value_loss"] - self.cfg.entropy_coef * terms["entropy"]
        with torch.no_grad():
            extra = torch.stack([(-log_ratio).mean(), ((ratio - 1).abs() > self.cfg.clip_ratio).float().mean()])
            vals = torch.stack([t.detach() for t in terms.values()] + list(extra)).tolist()  # one host read
        metrics = dict(batch.stats)
        metrics.update(zip(list(terms) + ["approx_kl", "clip_fraction"], vals))
        return loss, metrics

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        seeds = seeds_for(self.cfg.eval_seed, self.cfg.eval_episodes)
        m = aggregate_metrics(run_episodes(self.policy, self.env_cfg, seeds, rng_seed=self.cfg.eval_seed),
                              self.env_cfg)
        out = {k: m[k] for k in _EVAL_KEYS}
        out["primary"] = -m["value"]  # the trainer keeps the lowest primary
        return out

    def state(self) -> Dict[str, Any]:
        return {"model": self.net.state_dict()}

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.net.load_state_dict(state["model"])

    def model_spec(self) -> Dict[str, Any]:
        return {"family": "allocation_policy", "policy": self.net_cfg.to_dict(), "env": self.env_cfg.to_dict()}

    def tokenizer_meta(self):
        return None

    # ------------------------------------------------------------------ rollout
    @torch.no_grad()
    def _roll(self):
        n, T = self.cfg.episodes_per_rollout, self.env_cfg.horizon
        seq = self.policy.is_sequence
        traj = Trajectory.empty(T, n, self.device, self.net_cfg.window if seq else 0,
                                history_feature_dim(self.env_cfg.n_actions))
        venv = VectorEnv(self.env_cfg, n)
        obs = venv.reset([int(s) for s in self.rng.integers(0, 2 ** 31 - 1, size=n)])
        self._episodes_seen += n
        self.policy.start(n)
        clipped = 0
        for t in range(T):
            if seq:
                self.policy.hist.set_obs(obs)
                rows, lengths = self.policy.hist.ordered()
                traj.hist[t].copy_(torch.from_numpy(rows))
                traj.lengths[t].copy_(torch.from_numpy(lengths))
            traj.obs[t].copy_(torch.from_numpy(np.asarray(obs, dtype=np.float32)))
            logits, value = self.policy.evaluate(obs)
            logp_all = F.log_softmax(logits.float(), -1)
            a = torch.multinomial(logp_all.exp(), 1).squeeze(1)
            traj.actions[t], traj.logp[t], traj.values[t] = a, logp_all.gather(1, a[:, None]).squeeze(1), value
            a_host = a.cpu().numpy()
            obs, rewards, _, infos = venv.step(a_host)
            traj.rewards[t].copy_(torch.from_numpy(np.asarray(rewards, dtype=np.float32)))
            clipped += sum(i.clipped for i in infos)
            self.policy.observe(a_host, rewards, np.array([i.spend for i in infos]),
                                np.array([i.remaining_after for i in infos]))
        ep_value = traj.rewards.sum(0)
        stats = {"reward_mean": float(ep_value.mean()), "reward_std": float(ep_value.double().std(unbiased=False)),
                 "clipped_per_episode": clipped / n, "episodes_seen": float(self._episodes_seen),
                 "utilization": float((venv.cum_spend / self.env_cfg.budget).mean())}
        return traj, stats

    def _to_batch(self, traj: Trajectory, stats: Dict[str, float]) -> RolloutBatch:
        deltas = traj.rewards + self.cfg.gamma * traj.values[1:] - traj.values[:-1]
        adv = self._gae @ deltas
        ret = adv + traj.values[:-1]
        flat = lambda x: None if x is None else x.reshape(-1, *x.shape[2:])  # noqa: E731
        adv = flat(adv)
        if self.cfg.normalize_advantages and adv.numel() > 1:
            adv = (adv - adv.mean()) / (adv.std() + 1e-8)
        return RolloutBatch(flat(traj.obs), flat(traj.hist), flat(traj.lengths), flat(traj.actions),
                            flat(traj.logp), adv, flat(ret), torch.arange(adv.numel(), device=self.device), stats)


def build_allocation_ppo(params: Dict[str, Any], device: torch.device | str = "cpu") -> AllocationPPOAlgorithm:
    """From ``algorithm_params`` ``{env: {...}, policy: {...}, <AllocationPPOConfig fields>}``."""
    rest = {k: v for k, v in params.items() if k not in ("env", "policy")}
    return AllocationPPOAlgorithm(AllocationEnvConfig.from_dict(params.get("env") or {}),
                                  PolicyNetConfig.from_dict(params.get("policy") or {}),
                                  AllocationPPOConfig.from_dict(rest), device)


def load_allocation_policy(checkpoint: str, device: torch.device | str = "cpu") -> NeuralPolicy:
    """Rebuild the trained policy from a checkpoint directory written by the trainer."""
    from rl_project_b200.checkpoints.manager import CheckpointManager

    state = CheckpointManager.load(checkpoint, map_location="cpu")
    spec = state.model_spec or {}
    if spec.get("family") != "allocation_policy":
        raise ConfigError(f"checkpoint {checkpoint} is not an allocation policy "
                          f"(model_spec.family={spec.get('family')!r})")
    env_cfg = AllocationEnvConfig.from_dict(spec["env"])
    net = build_actor_critic(env_cfg.n_actions, PolicyNetConfig.from_dict(spec["policy"]))
    net.load_state_dict(state.model_state["model"])
    return NeuralPolicy(net.eval(), env_cfg, device)
