"""Actor-critic PPO over synthesis records (the tabular baseline of the synthesis domain).

Each record (encoded as a 128-d state) is a one-step episode.  The actor picks
one of 32 condition adjustments (4 temperature offsets x 4 time factors x 2
catalyst loadings) applied to the record's conditions; for molecules the
simulator knows, the outcomes of the adjusted conditions are predicted and
scored with ``reward_fn`` (the rule score), otherwise the record itself is
scored.  PPO proper: actions and their log-probabilities are sampled once per
mini-batch with the current policy, then ``ppo_epochs`` clipped-surrogate
updates with value MSE and an entropy bonus.  Metric keys follow
``src/forgeline/domains/synthesis/tabular_ppo.py:63-111``.
"""

from __future__ import annotations

import itertools
import json
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, Dict, List, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.errors import ConfigError, DatasetError
from rl_project_b200.domains.synthesis.constraints import validate_conditions
from rl_project_b200.domains.synthesis.features import STATE_DIM, encode_trajectory
from rl_project_b200.domains.synthesis.generator import MOLECULES, predict_outcomes
from rl_project_b200.domains.synthesis.reward import extract_outcomes, rule_score

ACTIONS: List[Tuple[float, float, float]] = list(itertools.product((-30.0, -10.0, 10.0, 30.0), (0.6, 1.0, 1.5, 2.2),
                                                                  (0.08, 0.2)))


def load_trajectories(path: str | Path) -> List[Dict[str, Any]]:
    path = Path(path)
    if not path.exists():
        raise DatasetError(f"trajectory file not found: {path}")
    with path.open() as fh:
        return [json.loads(line) for line in fh if line.strip()]


def apply_action(record: Dict[str, Any], action: int) -> Dict[str, Any]:
    """The record with conditions moved by ``ACTIONS[action]`` and outcomes re-predicted when possible."""
    dt, fh, cat = ACTIONS[action]
    o = extract_outcomes(record)
    cond, _ = validate_conditions({"temperature_celsius": o["temperature"] + dt, "time_hours": o["time"] * fh,
                                   "catalyst_loading_M": cat, "solvent_ratio_ml_mmol": o["solvent"]})
    out = dict(record)
    out["parameters"] = {**(record.get("parameters") or {}), **cond}
    if record.get("molecule") in MOLECULES:
        out["outcomes"] = predict_outcomes(record["molecule"], cond)
    return out


class TabularActorCritic(nn.Module):
    def __init__(self, state_dim: int = STATE_DIM, action_dim: int = len(ACTIONS), hidden_dim: int = 256):
        super().__init__()
        if min(state_dim, action_dim, hidden_dim) <= 0:
            raise ConfigError("dimensions must be positive")
        self.trunk = nn.Sequential(nn.Linear(state_dim, hidden_dim), nn.ReLU(), nn.Linear(hidden_dim, hidden_dim),
                                   nn.ReLU())
        self.pi = nn.Sequential(nn.Linear(hidden_dim, hidden_dim), nn.ReLU(), nn.Linear(hidden_dim, action_dim))
        self.v = nn.Sequential(nn.Linear(hidden_dim, hidden_dim), nn.ReLU(), nn.Linear(hidden_dim, 1))

    def forward(self, state: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """``(action probabilities [B, A], values [B, 1])``."""
        if state.dim() == 1:
            state = state.unsqueeze(0)
        h = self.trunk(state)
        return F.softmax(self.pi(h), dim=-1), self.v(h)


@dataclass
class TabularPPOConfig:
    learning_rate: float = 1e-4
    clip_ratio: float = 0.2
    epochs: int = 5
    batch_size: int = 8
    value_coef: float = 0.5
    entropy_coef: float = 0.01
    baseline_reward: float = 0.5
    ppo_epochs: int = 2
    seed: int = 0


class TabularPPOTrainer:
    def __init__(self, policy: TabularActorCritic, cfg: TabularPPOConfig,
                 reward_fn: Callable[[Dict[str, Any]], float] = rule_score, device: str = "cpu"):
        if cfg.learning_rate <= 0:
            raise ConfigError("learning_rate must be positive")
        self.policy = policy.to(device)
        self.cfg = cfg
        self.reward_fn = reward_fn
        self.device = device
        self.optimizer = torch.optim.Adam(self.policy.parameters(), lr=cfg.learning_rate)
        self.gen = torch.Generator().manual_seed(cfg.seed)

    def act(self, records: List[Dict[str, Any]], greedy: bool = True) -> List[int]:
        with torch.no_grad():
            probs, _ = self.policy(torch.stack([encode_trajectory(r) for r in records]).to(self.device))
        if greedy:
            return probs.argmax(-1).tolist()
        return torch.multinomial(probs.cpu(), 1, generator=self.gen).squeeze(1).tolist()

    def _update(self, states, actions, old_logp, rewards) -> Tuple[float, float, float]:
        c = self.cfg
        for _ in range(c.ppo_epochs):
            probs, values = self.policy(states)
            values = values.squeeze(-1)
            logp = torch.log(probs.gather(1, actions[:, None]).squeeze(1) + 1e-8)
            adv = rewards - values.detach()
            if adv.numel() > 1:
                adv = (adv - adv.mean()) / (adv.std() + 1e-8)
            ratio = torch.exp(logp - old_logp)
            policy_loss = -torch.min(ratio * adv, ratio.clamp(1 - c.clip_ratio, 1 + c.clip_ratio) * adv).mean()
            value_loss = F.mse_loss(values, rewards)
            entropy = -(probs * torch.log(probs + 1e-8)).sum(-1).mean()
            loss = policy_loss + c.value_coef * value_loss - c.entropy_coef * entropy
            self.optimizer.zero_grad()
            loss.backward()
            torch.nn.utils.clip_grad_norm_(self.policy.parameters(), 1.0)
            self.optimizer.step()
        return float(loss.detach()), float(policy_loss.detach()), float(value_loss.detach())

    def train(self, trajectories: List[Dict[str, Any]]) -> Dict[str, Any]:
        if not trajectories:
            raise DatasetError("empty trajectory list")
        self.policy.train()
        keys = ("epoch_rewards", "epoch_losses", "epoch_policy_losses", "epoch_value_losses")
        metrics: Dict[str, Any] = {k: [] for k in keys}
        for _ in range(self.cfg.epochs):
            acc = [0.0, 0.0, 0.0, 0.0]
            n = 0
            for i in range(0, len(trajectories), self.cfg.batch_size):
                batch = trajectories[i:i + self.cfg.batch_size]
                states = torch.stack([encode_trajectory(t) for t in batch]).to(self.device)
                with torch.no_grad():
                    probs, _ = self.policy(states)
                    actions = torch.multinomial(probs.cpu(), 1, generator=self.gen).squeeze(1).to(self.device)
                    old_logp = torch.log(probs.gather(1, actions[:, None]).squeeze(1) + 1e-8)
                rewards = torch.tensor([self.reward_fn(apply_action(t, int(a))) for t, a in zip(batch, actions.tolist())],
                                       dtype=torch.float32, device=self.device)
                loss, pl, vl = self._update(states, actions, old_logp, rewards)
                for j, v in enumerate((float(rewards.mean()), loss, pl, vl)):
                    acc[j] += v
                n += 1
            for k, v in zip(keys, acc):
                metrics[k].append(v / n)
        metrics["final_reward"] = metrics["epoch_rewards"][-1]
        metrics["improvement"] = (metrics["final_reward"] - self.cfg.baseline_reward) / self.cfg.baseline_reward * 100
        return metrics
