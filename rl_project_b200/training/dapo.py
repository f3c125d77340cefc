"""DAPO (the objective and options of ``src/forgeline/training/dapo.py``): clip-higher ratio bounds
``[1 - eps_low, 1 + eps_high]``, dynamic sampling (groups whose rewards have no variance are dropped),
a token-level loss normalised by the total response-token count of the batch, overlong reward shaping,
an optional KL term to a frozen reference and an optional full-distribution entropy bonus.

Because the loss is one sum over every response token of every active group, groups need not be scored
one by one: all trajectories of a micro-batch are packed into ONE right-padded ``[N, T]`` batch (row =
prompt + response, targets -1 outside the response) and scored in a single forward through the fused
LM-head log-prob kernel (entropy from the same pass).  Under causal attention the padding after a row
cannot change its log-probs.  The reference log-probs of the whole step come from one such pass in
``collect``.  Per-token values are kept response-aligned (``[rows, max response length]``).
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.core.protocols import RewardProvider, Trajectory
from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine
from rl_project_b200.rollouts.rewards.composite import batch_scores, score_trajectories
from rl_project_b200.training.common.advantages import group_relative_advantages
from rl_project_b200.training.common.logprobs import packed_response_logprobs
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm


@dataclass
class DAPOConfig:
    group_size: int = 4
    prompts_per_step: int = 2
    clip_eps_low: float = 0.2
    clip_eps_high: float = 0.28
    kl_coef: float = 0.04
    entropy_coef: float = 0.0
    dynamic_sampling: bool = True
    overlong_penalty: float = -1.0
    max_response_len: Optional[int] = None
    seed: int = 0

    def validate(self) -> None:
        if self.group_size < 2:
            raise ConfigError("DAPO group_size must be >= 2")
        if not (0 < self.clip_eps_low < 1 and 0 < self.clip_eps_high < 1):
            raise ConfigError("clip epsilons must be in (0, 1)")
        if self.clip_eps_high < self.clip_eps_low:
            raise ConfigError("clip_eps_high must be >= clip_eps_low (clip-higher)")


@dataclass
class DAPOGroup:
    trajectories: List[Trajectory]
    rewards: torch.Tensor
    advantages: torch.Tensor
    old_logprobs: torch.Tensor  # [G, R] response-aligned
    ref_logprobs: torch.Tensor  # [G, R] response-aligned (zeros without a KL term)
    mask: torch.Tensor  # [G, R]
    skipped: bool = False


def dapo_token_objective(ratio: torch.Tensor, adv: torch.Tensor, eps_low: float, eps_high: float) -> torch.Tensor:
    """Elementwise ``-min(r A, clip(r, 1 - eps_low, 1 + eps_high) A)``."""
    return -torch.minimum(ratio * adv, ratio.clamp(1.0 - eps_low, 1.0 + eps_high) * adv)


def _response_mask(trajs: Sequence[Trajectory], width: int) -> torch.Tensor:
    lengths = torch.tensor([t.response_length for t in trajs])
    return (torch.arange(width)[None, :] < lengths[:, None]).float()


def _recorded(trajs: Sequence[Trajectory], width: int) -> torch.Tensor:
    out = torch.zeros(len(trajs), width)
    for i, t in enumerate(trajs):
        if t.old_logprobs is not None:
            out[i, :t.old_logprobs.numel()] = t.old_logprobs.float()
    return out


def _pad_cols(x: torch.Tensor, width: int) -> torch.Tensor:
    return x if x.shape[1] == width else torch.nn.functional.pad(x, (0, width - x.shape[1]))


class DAPOAlgorithm(PostTrainingAlgorithm):
    name = "dapo"

    def __init__(self, policy, prompts: Sequence[torch.Tensor], reward: RewardProvider, config: DAPOConfig,
                 rollout: Optional[RolloutConfig] = None, tasks: Optional[Sequence[Dict[str, Any]]] = None):
        config.validate()
        self.policy, self.cfg, self.reward = policy, config, reward
        self.prompts = list(prompts)
        self.tasks = list(tasks) if tasks else [{} for _ in self.prompts]
        rc = rollout or RolloutConfig()
        rc.group_size = config.group_size
        self.rollouts = RolloutEngine(policy, rc)
        self.max_response_len = config.max_response_len or rc.max_new_tokens
        if config.kl_coef > 0 and not policy.has_adapter and policy.reference_model is None:
            policy.with_frozen_reference()
        self.rng = random.Random(config.seed)
        self._last_stats: Dict[str, float] = {}

    def parameters(self) -> List[nn.Parameter]:
        return self.policy.trainable_parameters()

    def modules(self):
        return (self.policy.model,)

    def frozen_modules(self):
        return (self.policy.reference_model,) if self.policy.reference_model is not None else ()

    def _score(self, trajs: Sequence[Trajectory], width: int, entropy: bool = False):
        return packed_response_logprobs(self.policy, trajs, width, entropy)

    # ------------------------------------------------------------ collection
    def _shape_rewards(self, trajs: Sequence[Trajectory], rewards: torch.Tensor) -> torch.Tensor:
        """Overlong shaping: a response at the length budget gets ``overlong_penalty`` times its overshoot."""
        for g, t in enumerate(trajs):
            if t.response_length >= self.max_response_len:
                rewards[g] += self.cfg.overlong_penalty * max(0.0, t.response_length / self.max_response_len - 1.0)
                t.truncated = True
        return rewards

    @torch.no_grad()
    def collect(self, step: int) -> List[DAPOGroup]:
        picks = [self.rng.randrange(len(self.prompts)) for _ in range(self.cfg.prompts_per_step)]
        traj_groups = self.rollouts.rollout_many([self.prompts[i] for i in picks], [self.tasks[i] for i in picks])
        groups = []
        for trajs in traj_groups:
            rewards = self._shape_rewards(trajs, torch.tensor(score_trajectories(self.reward, trajs),
                                                              dtype=torch.float32))
            R = max(t.response_length for t in trajs)
            mask = _response_mask(trajs, R)
            skipped = self.cfg.dynamic_sampling and float(rewards.std()) < 1e-6
            groups.append(DAPOGroup(trajs, rewards, group_relative_advantages(rewards, clamp_std=True),
                                    _recorded(trajs, R) * mask, torch.zeros(len(trajs), R), mask, skipped))
        live = [g for g in groups if not g.skipped]
        flat = [t for g in live for t in g.trajectories]
        if flat:
            R = max(t.response_length for t in flat)
            if not all(t.old_logprobs is not None for t in flat):  # the rollout did not record them
                old, _ = self._score(flat, R)
                self._split(live, old.cpu(), "old_logprobs")
            if self.cfg.kl_coef > 0:
                with self.policy.reference():
                    ref, _ = self._score(flat, R)
                self._split(live, ref.cpu(), "ref_logprobs")
        rewards = torch.cat([g.rewards for g in groups])
        n_skip = sum(g.skipped for g in groups)
        self._last_stats = {"reward_mean": float(rewards.mean()), "groups_skipped": float(n_skip),
                            "active_groups": float(len(groups) - n_skip),
                            "truncated": float(sum(t.truncated for g in groups for t in g.trajectories))}
        return groups

    @staticmethod
    def _split(groups: Sequence[DAPOGroup], values: torch.Tensor, field_name: str) -> None:
        row = 0
        for g in groups:
            n, R = g.mask.shape
            setattr(g, field_name, values[row:row + n, :R] * g.mask)
            row += n

    # ------------------------------------------------------------ objective
    def loss(self, groups: List[DAPOGroup], micro_step: int, n_micro: int):
        chunk = [g for g in (groups[micro_step::n_micro] if n_micro > 1 else groups) if not g.skipped]
        ntok = float(sum(float(g.mask.sum()) for g in chunk))
        if ntok == 0:
            zero = sum(p.sum() for p in self.parameters()) * 0.0
            return zero, {**self._last_stats, "policy_loss": 0.0, "kl": 0.0, "entropy": 0.0, "tokens": 0.0}
        dev = self.policy.device
        trajs = [t for g in chunk for t in g.trajectories]
        R = max(g.mask.shape[1] for g in chunk)
        cat = lambda name: torch.cat([_pad_cols(getattr(g, name), R) for g in chunk]).to(dev)  # noqa: E731
        mask, old, ref = cat("mask"), cat("old_logprobs"), cat("ref_logprobs")
        adv = torch.cat([g.advantages for g in chunk]).to(dev)[:, None]
        new, ent_tok = self._score(trajs, R, entropy=self.cfg.entropy_coef > 0)
        new = new * mask
        per_tok = dapo_token_objective(torch.exp(new - old) * mask, adv, self.cfg.clip_eps_low, self.cfg.clip_eps_high)
        pg = (per_tok * mask).sum()
        kl = ((new - ref) * mask).sum() if self.cfg.kl_coef > 0 else torch.zeros((), device=dev)
        ent = (ent_tok * mask).sum() if ent_tok is not None else torch.zeros((), device=dev)
        loss = (pg + self.cfg.kl_coef * kl - self.cfg.entropy_coef * ent) / ntok
        return loss, {**self._last_stats, "policy_loss": pg.detach() / ntok, "kl": kl.detach() / ntok,
                      "entropy": ent.detach() / ntok, "tokens": ntok}

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        n = min(8, len(self.prompts))
        if n == 0:
            return {"reward": 0.0, "pass_rate": 0.0}
        groups = self.rollouts.rollout_many(self.prompts[:n], self.tasks[:n], group_size=1)  # one batched decode
        results = batch_scores(self.reward, [g[0] for g in groups])
        return {"reward": sum(r.value for r in results) / n, "pass_rate": sum(bool(r.passed) for r in results) / n}

    def state(self) -> Dict[str, Any]:
        return self.policy.state_for_checkpoint()

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.policy.load_checkpoint_state(state)

    def model_spec(self) -> Dict[str, Any]:
        return self.policy.spec.to_dict()

    def tokenizer_meta(self):
        return self.policy.tokenizer.metadata()
