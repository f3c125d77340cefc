"""Allocation policies behind one batched interface.

``act(obs [n, 14], ctx: StepArrays, rng, greedy) -> (actions [n], probs [n, A])``;
``observe(actions, rewards, spends, remaining)`` feeds back the realised step;
``action_probs(obs, ctx)`` gives the target-policy distribution for off-policy
evaluation without sampling or changing state.

Baselines (``src/forgeline/domains/allocation/policies.py:82-165`` behaviour):
a value-per-cost threshold pacer, and a primal-dual pacer whose price follows
projected subgradient steps on the per-step budget rate.  Learned: MLP and GRU
actor-critics (the GRU reads a window of realised history, from which the
latent pressure can be inferred); an epsilon-mix wrapper for logging policies.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from typing import Any, Dict, Optional, Tuple

import numpy as np
import torch
import torch.nn as nn

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.domains.allocation.env import (OBS_DIM, AllocationEnvConfig, StepArrays,  # noqa: F401
                                                     StepContext, strict_config)


def one_hot(actions: np.ndarray, n: int) -> np.ndarray:
    out = np.zeros((len(actions), n))
    out[np.arange(len(actions)), np.asarray(actions, dtype=np.int64)] = 1.0
    return out


class Policy:
    name = "policy"
    stochastic = False

    def start(self, n: int) -> None:
        pass

    def act(self, obs: np.ndarray, ctx: StepArrays, rng: np.random.Generator, greedy: bool = False):
        raise NotImplementedError

    def observe(self, actions, rewards, spends, remaining=None) -> None:
        pass

    def action_probs(self, obs: np.ndarray, ctx: StepArrays) -> np.ndarray:
        raise NotImplementedError


class _Deterministic(Policy):
    def decide(self, ctx: StepArrays) -> np.ndarray:
        raise NotImplementedError

    def act(self, obs, ctx, rng, greedy=False):
        a = self.decide(ctx)
        return a, one_hot(a, self.cfg.n_actions)

    def action_probs(self, obs, ctx):
        return one_hot(self.decide(ctx), self.cfg.n_actions)


class ThresholdPacingPolicy(_Deterministic):
    """Allocate at ``level`` when value x quality / cost >= threshold and spend is on the pro-rata pace."""

    name = "threshold_pacing"

    def __init__(self, env_cfg: AllocationEnvConfig, threshold: float = 1.0, level: int = 2,
                 pacing_slack: float = 0.05):
        if not 0 < level < env_cfg.n_actions:
            raise ConfigError("level must be a non-abstain action index")
        self.cfg, self.threshold, self.level, self.slack = env_cfg, threshold, level, pacing_slack

    def decide(self, c: StepArrays) -> np.ndarray:
        good = c.value * c.quality / np.maximum(c.cost, 1e-9) >= self.threshold
        on_pace = c.cum_spend <= c.budget * (c.t / c.horizon + self.slack)
        return np.where(good & on_pace & (c.remaining > 0), self.level, 0)


class DualPacingPolicy(_Deterministic):
    """Lagrangian pacer: a = argmax_m v q g(m) - lambda m c, with lambda <- max(0, lambda + lr (x - B/T))."""

    name = "dual_pacing"

    def __init__(self, env_cfg: AllocationEnvConfig, learning_rate: float = 0.2, initial_price: float = 0.8):
        if learning_rate <= 0 or initial_price < 0:
            raise ConfigError("dual pacing needs learning_rate > 0 and initial_price >= 0")
        self.cfg, self.lr, self.lam0 = env_cfg, learning_rate, initial_price
        self.M = np.asarray(env_cfg.multipliers)
        self.lam = np.zeros(0)
        self.rate = env_cfg.budget / env_cfg.horizon

    def start(self, n: int) -> None:
        self.lam = np.full(n, float(self.lam0))

    def decide(self, c: StepArrays) -> np.ndarray:
        if self.lam.shape[0] != len(c.value):
            self.start(len(c.value))
        gain = (c.value * c.quality)[:, None] * (1.0 - np.exp(-self.M))[None, :]
        score = gain - self.lam[:, None] * self.M[None, :] * c.cost[:, None]
        return np.where(c.remaining > 0, score.argmax(1), 0)

    def observe(self, actions, rewards, spends, remaining=None) -> None:
        self.lam = np.maximum(0.0, self.lam + self.lr * (np.asarray(spends) - self.rate))

    def prices(self) -> np.ndarray:
        return self.lam.copy()


@dataclass
class PolicyNetConfig:
    kind: str = "mlp"  # mlp | gru
    hidden: int = 64
    window: int = 8
    gru_layers: int = 1

    def validate(self) -> None:
        if self.kind not in ("mlp", "gru"):
            raise ConfigError("policy kind must be mlp|gru")
        if self.hidden < 1 or self.window < 2 or self.gru_layers < 1:
            raise ConfigError("hidden >= 1, window >= 2, gru_layers >= 1 required")

    @classmethod
    def from_dict(cls, d: Dict[str, Any]) -> "PolicyNetConfig":
        return strict_config(cls, d, "policy")

    def to_dict(self) -> Dict[str, Any]:
        return dataclasses.asdict(self)


def history_feature_dim(n_actions: int) -> int:
    """obs, one-hot action, reward / v_mean, spend / c_mean, remaining / budget."""
    return OBS_DIM + n_actions + 3


class ActorCritic(nn.Module):
    kind = "base"

    def __init__(self, n_actions: int, config: PolicyNetConfig):
        super().__init__()
        self.n_actions, self.config = n_actions, config


class MLPActorCritic(ActorCritic):
    kind = "mlp"

    def __init__(self, n_actions: int, config: PolicyNetConfig):
        super().__init__(n_actions, config)
        h = config.hidden
        self.body = nn.Sequential(nn.Linear(OBS_DIM, h), nn.Tanh(), nn.Linear(h, h), nn.Tanh())
        self.pi, self.v = nn.Linear(h, n_actions), nn.Linear(h, 1)

    def forward(self, obs: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        z = self.body(obs)
        return self.pi(z), self.v(z).squeeze(-1)


class GRUActorCritic(ActorCritic):
    """GRU over the last ``window`` realised steps (oldest first, zero rows before the episode start are
    skipped by packing), concatenated with the current observation."""

    kind = "gru"

    def __init__(self, n_actions: int, config: PolicyNetConfig):
        super().__init__(n_actions, config)
        h = config.hidden
        self.gru = nn.GRU(history_feature_dim(n_actions), h, num_layers=config.gru_layers, batch_first=True)
        self.obs_proj = nn.Linear(OBS_DIM, h)
        self.head = nn.Sequential(nn.Linear(2 * h, h), nn.Tanh())
        self.pi, self.v = nn.Linear(h, n_actions), nn.Linear(h, 1)

    def forward(self, features) -> Tuple[torch.Tensor, torch.Tensor]:
        obs, hist, lengths = features  # [n, 14], [n, W, D] (valid rows first), [n]
        n = obs.shape[0]
        enc = obs.new_zeros(n, self.gru.hidden_size)
        has = lengths > 0
        if bool(has.any()):
            packed = nn.utils.rnn.pack_padded_sequence(hist[has], lengths[has].cpu(), batch_first=True,
                                                       enforce_sorted=False)
            _, h_n = self.gru(packed)
            enc = enc.index_put((has.nonzero().squeeze(1),), h_n[-1])
        z = self.head(torch.cat([torch.tanh(self.obs_proj(obs)), enc], -1))
        return self.pi(z), self.v(z).squeeze(-1)


def build_actor_critic(n_actions: int, config: PolicyNetConfig) -> ActorCritic:
    config.validate()
    return (MLPActorCritic if config.kind == "mlp" else GRUActorCritic)(n_actions, config)


class HistoryBuffer:
    """Per-episode window of realised steps kept as a ring: ``push`` writes each episode's new row into its next
    slot (no shifting of the window); ``ordered`` returns the rows oldest-first with the valid ones at the front
    and zeros after, the layout the GRU packs."""

    def __init__(self, n: int, window: int, n_actions: int, env_cfg: AllocationEnvConfig):
        self.n, self.window, self.n_actions, self.cfg = n, window, n_actions, env_cfg
        self.dim = history_feature_dim(n_actions)
        self.ring = np.zeros((n, window, self.dim), dtype=np.float32)
        self.count = np.zeros(n, dtype=np.int64)  # rows pushed so far per episode
        self._norm = np.array([env_cfg.value_mean, env_cfg.cost_mean, env_cfg.budget], dtype=np.float64)
        self._obs: Optional[np.ndarray] = None

    @property
    def lengths(self) -> np.ndarray:
        return np.minimum(self.count, self.window)

    def set_obs(self, obs: np.ndarray) -> None:
        self._obs = np.asarray(obs, dtype=np.float32)

    def push(self, actions, rewards, spends, remaining) -> None:
        """Row = (observation before the step, one-hot action, reward / v_mean, spend / c_mean, remaining / B)."""
        ep = np.arange(self.n)
        row = np.zeros((self.n, self.dim), dtype=np.float32)
        row[:, :OBS_DIM] = self._obs
        row[ep, OBS_DIM + np.asarray(actions, dtype=np.int64)] = 1.0
        row[:, -3:] = np.stack([np.asarray(rewards), np.asarray(spends), np.asarray(remaining)], 1) / self._norm
        self.ring[ep, self.count % self.window] = row
        self.count += 1

    def ordered(self) -> Tuple[np.ndarray, np.ndarray]:
        L = self.lengths
        slots = (self.count - L)[:, None] + np.arange(self.window)[None, :]  # oldest kept row first
        out = np.take_along_axis(self.ring, (slots % self.window)[:, :, None], axis=1)
        out[np.arange(self.window)[None, :] >= L[:, None]] = 0.0
        return out, L

    @property
    def buf(self) -> np.ndarray:
        return self.ordered()[0]

    def tensors(self, device) -> Tuple[torch.Tensor, torch.Tensor]:
        rows, L = self.ordered()
        return torch.as_tensor(rows, device=device), torch.as_tensor(L, device=device)


class NeuralPolicy(Policy):
    stochastic = True

    def __init__(self, net: ActorCritic, env_cfg: AllocationEnvConfig, device: torch.device | str = "cpu"):
        self.net, self.cfg = net.to(device), env_cfg
        self.device = torch.device(device)
        self.name = f"ppo_{net.kind}"
        self.hist: Optional[HistoryBuffer] = None

    @property
    def is_sequence(self) -> bool:
        return self.net.kind == "gru"

    def start(self, n: int) -> None:
        self.hist = HistoryBuffer(n, self.net.config.window, self.cfg.n_actions, self.cfg) if self.is_sequence else None

    def features(self, obs: np.ndarray):
        o = torch.as_tensor(np.asarray(obs, dtype=np.float32), device=self.device)
        if not self.is_sequence:
            return o
        if self.hist is None or self.hist.n != o.shape[0]:
            self.start(o.shape[0])
        h, lens = self.hist.tensors(self.device)
        return o, h, lens

    @torch.no_grad()
    def evaluate(self, obs: np.ndarray):
        return self.net(self.features(obs))

    def act(self, obs, ctx, rng, greedy=False):
        if self.is_sequence:
            if self.hist is None or self.hist.n != len(obs):
                self.start(len(obs))
            self.hist.set_obs(obs)
        logits, _ = self.evaluate(obs)
        probs = torch.softmax(logits.double(), -1).cpu().numpy()
        if greedy:
            return probs.argmax(1), probs
        u = rng.uniform(size=(len(obs), 1))
        return np.minimum((u > probs.cumsum(1)).sum(1), probs.shape[1] - 1), probs

    def observe(self, actions, rewards, spends, remaining=None) -> None:
        if self.is_sequence and self.hist is not None:
            rem = remaining if remaining is not None else np.zeros(len(actions))
            self.hist.push(actions, rewards, spends, rem)

    def action_probs(self, obs, ctx):
        logits, _ = self.evaluate(obs)
        return torch.softmax(logits.double(), -1).cpu().numpy()


class EpsilonMixPolicy(Policy):
    """``(1 - eps) base + eps uniform``: a logging policy with full support (needed for OPE)."""

    stochastic = True

    def __init__(self, base: Policy, epsilon: float, n_actions: int):
        if not 0.0 <= epsilon <= 1.0:
            raise ConfigError("epsilon must be in [0, 1]")
        self.base, self.eps, self.n_actions = base, epsilon, n_actions
        self.name = f"{base.name}+eps{epsilon:g}"

    def start(self, n):
        self.base.start(n)

    def _mix(self, probs: np.ndarray) -> np.ndarray:
        return (1.0 - self.eps) * probs + self.eps / self.n_actions

    def act(self, obs, ctx, rng, greedy=False):
        _, p = self.base.act(obs, ctx, rng, greedy=True)
        mixed = self._mix(p)
        if greedy:
            return mixed.argmax(1), mixed
        u = rng.uniform(size=(len(obs), 1))
        return np.minimum((u > mixed.cumsum(1)).sum(1), self.n_actions - 1), mixed

    def observe(self, actions, rewards, spends, remaining=None):
        self.base.observe(actions, rewards, spends, remaining)

    def action_probs(self, obs, ctx):
        return self._mix(self.base.action_probs(obs, ctx))


def policy_spec(policy: Policy) -> Dict[str, Any]:
    spec: Dict[str, Any] = {"name": policy.name, "stochastic": policy.stochastic}
    for attr in ("threshold", "level", "slack", "lr", "lam0", "eps"):
        if hasattr(policy, attr):
            spec[attr] = getattr(policy, attr)
    if isinstance(policy, NeuralPolicy):
        spec["net"] = policy.net.config.to_dict()
    return spec
