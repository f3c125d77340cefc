"""PPO for allocation policies, run by the framework's ``Trainer`` (algorithm ``allocation_ppo``).

``collect`` rolls out ``episodes_per_rollout`` episodes in one vectorised
environment (a fresh rollout every ``ppo_epochs`` optimiser steps, reshuffled
minibatches in between); advantages are per-episode GAE (gamma = 1 by default:
undiscounted finite horizon), computed for all episodes at once.  The loss is
the clipped surrogate + value MSE - entropy bonus.  ``evaluate`` runs the
stochastic policy on a held-out seed family; ``primary`` = -value so the
trainer keeps the best checkpoint.  The checkpoint ``model_spec`` has
``family: allocation_policy`` plus the env and network configs, from which
``load_allocation_policy`` rebuilds the policy (the spec layout follows
``src/forgeline/domains/allocation/ppo.py:190-217``).
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.domains.allocation.env import OBS_DIM, AllocationEnvConfig, VectorEnv
from rl_project_b200.domains.allocation.policies import (NeuralPolicy, PolicyNetConfig, build_actor_critic,
                                                         history_feature_dim)
from rl_project_b200.domains.allocation.rollout import aggregate_metrics, run_episodes, seeds_for
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm
from rl_project_b200.training.ppo import ppo_clipped_objective


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
        if min(self.episodes_per_rollout, self.ppo_epochs, self.eval_episodes) < 1:
            raise ConfigError("episodes_per_rollout, ppo_epochs and eval_episodes must be >= 1")
        if not (0 < self.clip_ratio < 1 and 0 < self.gamma <= 1 and 0 <= self.gae_lambda <= 1):
            raise ConfigError("clip_ratio in (0,1), gamma in (0,1], gae_lambda in [0,1] required")

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "AllocationPPOConfig":
        unknown = set(d) - {f.name for f in dataclasses.fields(cls)}
        if unknown:
            raise ConfigError(f"unknown AllocationPPOConfig keys: {sorted(unknown)}")
        c = cls(**d)
        c.validate()
        return c


def batched_gae(rewards: np.ndarray, values: np.ndarray, gamma: float, lam: float):
    """GAE over ``[T, n]`` rewards and ``[T+1, n]`` values (terminal value 0): (advantages, returns)."""
    T = rewards.shape[0]
    adv = np.zeros_like(rewards)
    run = np.zeros(rewards.shape[1], dtype=rewards.dtype)
    for t in range(T - 1, -1, -1):
        run = rewards[t] + gamma * values[t + 1] - values[t] + gamma * lam * run
        adv[t] = run
    return adv, adv + values[:T]


@dataclass
class RolloutBatch:
    obs: torch.Tensor
    hist: Optional[torch.Tensor]
    lengths: Optional[torch.Tensor]
    actions: torch.Tensor
    old_logp: torch.Tensor
    advantages: torch.Tensor
    returns: torch.Tensor
    perm: torch.Tensor
    stats: Dict[str, float]


class AllocationPPOAlgorithm(PostTrainingAlgorithm):
    name = "allocation_ppo"

    def __init__(self, env_cfg: AllocationEnvConfig, net_cfg: PolicyNetConfig, config: AllocationPPOConfig,
                 device: torch.device | str = "cpu"):
        env_cfg.validate()
        net_cfg.validate()
        config.validate()
        self.env_cfg, self.net_cfg, self.cfg = env_cfg, net_cfg, config
        self.device = torch.device(device)
        self.net = build_actor_critic(env_cfg.n_actions, net_cfg).to(self.device)
        self.policy = NeuralPolicy(self.net, env_cfg, self.device)
        self.rng = np.random.default_rng(config.seed)
        self._batch: Optional[RolloutBatch] = None
        self._episodes_seen = 0

    def parameters(self) -> List[nn.Parameter]:
        return [p for p in self.net.parameters() if p.requires_grad]

    def modules(self):
        return (self.net,)

    def collect(self, step: int) -> RolloutBatch:
        if self._batch is None or step % self.cfg.ppo_epochs == 0:
            self._batch = self._rollout()
        S = self._batch.actions.shape[0]
        self._batch.perm = torch.as_tensor(self.rng.permutation(S), device=self.device)
        return self._batch

    @torch.no_grad()
    def _rollout(self) -> RolloutBatch:
        cfg, env_cfg = self.cfg, self.env_cfg
        n, T = cfg.episodes_per_rollout, env_cfg.horizon
        seeds = [int(s) for s in self.rng.integers(0, 2 ** 31 - 1, size=n)]
        self._episodes_seen += n
        venv = VectorEnv(env_cfg, n)
        obs = venv.reset(seeds)
        self.policy.start(n)
        seq = self.policy.is_sequence
        W, D = self.net_cfg.window, history_feature_dim(env_cfg.n_actions)
        obs_buf = np.zeros((T, n, OBS_DIM), np.float32)
        hist_buf = np.zeros((T, n, W, D), np.float32) if seq else None
        len_buf = np.zeros((T, n), np.int64)
        act_buf = np.zeros((T, n), np.int64)
        logp_buf = np.zeros((T, n), np.float32)
        val_buf = np.zeros((T + 1, n), np.float32)
        rew_buf = np.zeros((T, n), np.float32)
        clipped = 0
        for t in range(T):
            if seq:
                self.policy.hist.set_obs(obs)
                hist_buf[t], len_buf[t] = self.policy.hist.buf, self.policy.hist.lengths
            logits, value = self.policy.evaluate(obs)
            dist = torch.distributions.Categorical(logits=logits)
            a = dist.sample()
            obs_buf[t], act_buf[t] = obs, a.cpu().numpy()
            logp_buf[t], val_buf[t] = dist.log_prob(a).cpu().numpy(), value.cpu().numpy()
            obs, rewards, _, infos = venv.step(act_buf[t])
            rew_buf[t] = rewards
            clipped += sum(i.clipped for i in infos)
            self.policy.observe(act_buf[t], rewards, np.array([i.spend for i in infos]),
                                np.array([i.remaining_after for i in infos]))
        adv, ret = batched_gae(rew_buf, val_buf, cfg.gamma, cfg.gae_lambda)
        flat = lambda x: torch.as_tensor(x.reshape(T * n, *x.shape[2:]), device=self.device)  # noqa: E731
        advantages = flat(adv)
        if cfg.normalize_advantages and advantages.numel() > 1:
            advantages = (advantages - advantages.mean()) / (advantages.std() + 1e-8)
        ep_values = rew_buf.sum(0)
        stats = {"reward_mean": float(ep_values.mean()), "reward_std": float(ep_values.std()),
                 "clipped_per_episode": clipped / n, "episodes_seen": float(self._episodes_seen),
                 "utilization": float((venv.cum_spend / env_cfg.budget).mean())}
        return RolloutBatch(flat(obs_buf), flat(hist_buf) if seq else None, flat(len_buf) if seq else None,
                            flat(act_buf), flat(logp_buf), advantages, flat(ret), torch.arange(T * n), stats)

    def loss(self, batch: RolloutBatch, micro_step: int, n_micro: int):
        idx = batch.perm[micro_step::n_micro] if n_micro > 1 else batch.perm
        feats = batch.obs[idx] if batch.hist is None else (batch.obs[idx], batch.hist[idx], batch.lengths[idx])
        logits, values = self.net(feats)
        logp_all = F.log_softmax(logits, -1)
        logp = logp_all.gather(1, batch.actions[idx, None]).squeeze(1)
        ratio = torch.exp(logp - batch.old_logp[idx])
        pg = ppo_clipped_objective(ratio, batch.advantages[idx], self.cfg.clip_ratio).mean()
        v_loss = F.mse_loss(values, batch.returns[idx])
        entropy = -(logp_all.exp() * logp_all).sum(-1).mean()
        loss = pg + self.cfg.value_coef * v_loss - self.cfg.entropy_coef * entropy
        with torch.no_grad():
            metrics = {**batch.stats, "policy_loss": float(pg), "value_loss": float(v_loss), "entropy": float(entropy),
                       "approx_kl": float((batch.old_logp[idx] - logp).mean()),
                       "clip_fraction": float(((ratio - 1).abs() > self.cfg.clip_ratio).float().mean())}
        return loss, metrics

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        eps = run_episodes(self.policy, self.env_cfg, seeds_for(self.cfg.eval_seed, self.cfg.eval_episodes),
                           rng_seed=self.cfg.eval_seed)
        m = aggregate_metrics(eps, self.env_cfg)
        out = {k: m[k] for k in ("value", "value_std", "utilization", "pacing_error", "early_exhaustion",
                                 "violations", "final_pressure")}
        out["primary"] = -m["value"]
        return out

    def state(self) -> Dict[str, Any]:
        return {"model": self.net.state_dict()}

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.net.load_state_dict(state["model"])

    def model_spec(self) -> Dict[str, Any]:
        return {"family": "allocation_policy", "policy": self.net_cfg.to_dict(), "env": self.env_cfg.to_dict()}

    def tokenizer_meta(self):
        return None


def build_allocation_ppo(params: Dict[str, Any], device: torch.device | str = "cpu") -> AllocationPPOAlgorithm:
    """From ``algorithm_params`` ``{env: {...}, policy: {...}, <AllocationPPOConfig fields>}``."""
    p = dict(params)
    env_cfg = AllocationEnvConfig.from_dict(p.pop("env", {}) or {})
    net_cfg = PolicyNetConfig.from_dict(p.pop("policy", {}) or {})
    return AllocationPPOAlgorithm(env_cfg, net_cfg, AllocationPPOConfig.from_dict(p), device)


def load_allocation_policy(checkpoint: str, device: torch.device | str = "cpu") -> NeuralPolicy:
    from rl_project_b200.checkpoints.manager import CheckpointManager

    state = CheckpointManager.load(checkpoint, map_location="cpu")
    spec = state.model_spec or {}
    if spec.get("family") != "allocation_policy":
        raise ConfigError(f"checkpoint {checkpoint} is not an allocation policy "
                          f"(model_spec.family={spec.get('family')!r})")
    env_cfg = AllocationEnvConfig.from_dict(spec["env"])
    net = build_actor_critic(env_cfg.n_actions, PolicyNetConfig.from_dict(spec["policy"]))
    net.load_state_dict(state.model_state["model"])
    net.eval()
    return NeuralPolicy(net, env_cfg, device)
