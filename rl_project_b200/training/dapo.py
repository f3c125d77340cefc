"""DAPO (``src/forgeline/training/dapo.py`` objective): clip-higher bounds
``[1 - eps_low, 1 + eps_high]``, dynamic sampling (zero-variance groups
dropped), token-level loss normalised by the total response-token count,
overlong reward shaping and an optional full-distribution entropy bonus
(computed by the fused LM-head entropy kernel)."""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional, Sequence

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.core.protocols import RewardProvider, Trajectory
from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine, stack_group, stack_old_logprobs
from rl_project_b200.rollouts.rewards.composite import score_trajectories
from rl_project_b200.training.common.advantages import group_relative_advantages
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
    old_logprobs: torch.Tensor
    ref_logprobs: torch.Tensor
    mask: torch.Tensor
    skipped: bool = False


def dapo_token_objective(ratio: torch.Tensor, adv: torch.Tensor, eps_low: float, eps_high: float) -> torch.Tensor:
    return -torch.min(ratio * adv, torch.clamp(ratio, 1.0 - eps_low, 1.0 + eps_high) * adv)


class DAPOAlgorithm(PostTrainingAlgorithm):
    name = "dapo"

    def __init__(self, policy, prompts: Sequence[torch.Tensor], reward: RewardProvider, config: DAPOConfig,
                 rollout: Optional[RolloutConfig] = None, tasks: Optional[Sequence[Dict[str, Any]]] = None):
        config.validate()
        self.policy = policy
        self.cfg = config
        self.reward = reward
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

    @torch.no_grad()
    def collect(self, step: int) -> List[DAPOGroup]:
        idx = [self.rng.randrange(len(self.prompts)) for _ in range(self.cfg.prompts_per_step)]
        groups, skipped = [], 0
        for trajs in self.rollouts.rollout_many([self.prompts[i] for i in idx], [self.tasks[i] for i in idx]):
            rewards = torch.tensor(score_trajectories(self.reward, trajs), dtype=torch.float32)
            for g, t in enumerate(trajs):
                if t.response_length >= self.max_response_len:
                    rewards[g] += self.cfg.overlong_penalty * max(0.0, t.response_length / self.max_response_len - 1.0)
                    t.truncated = True
            prompt, resp, mask = stack_group(trajs, self.policy.pad_token_id)
            if all(t.old_logprobs is not None for t in trajs):
                old = stack_old_logprobs(trajs, resp.shape[1]) * mask
            else:
                old = self.policy.logprobs(prompt, resp).float().cpu() * mask
            if self.cfg.kl_coef > 0:
                with self.policy.reference():
                    ref = self.policy.logprobs(prompt, resp).float().cpu() * mask
            else:
                ref = torch.zeros_like(old)
            grp = DAPOGroup(trajs, rewards, group_relative_advantages(rewards, clamp_std=True), old, ref, mask)
            if self.cfg.dynamic_sampling and float(rewards.std()) < 1e-6:
                grp.skipped = True
                skipped += 1
            groups.append(grp)
        all_r = torch.cat([g.rewards for g in groups])
        self._last_stats = {"reward_mean": float(all_r.mean()), "groups_skipped": float(skipped),
                            "active_groups": float(len(groups) - skipped),
                            "truncated": float(sum(t.truncated for g in groups for t in g.trajectories))}
        return groups

    def loss(self, groups: List[DAPOGroup], micro_step: int, n_micro: int):
        chunk = groups[micro_step::n_micro] if n_micro > 1 else groups
        dev = self.policy.device
        pg = torch.zeros((), device=dev)
        kl = torch.zeros((), device=dev)
        ent = torch.zeros((), device=dev)
        ntok = 0.0
        for grp in chunk:
            if grp.skipped:
                continue
            prompt, resp, _ = stack_group(grp.trajectories, self.policy.pad_token_id)
            mask = grp.mask.to(dev)
            if self.cfg.entropy_coef > 0:
                new, ent_tok = self.policy.logprobs_with_entropy(prompt, resp)
                ent = ent + (ent_tok.float() * mask).sum()
            else:
                new = self.policy.logprobs(prompt, resp)
            new = new.float() * mask
            ratio = torch.exp(new - grp.old_logprobs.to(dev)) * mask
            per_tok = dapo_token_objective(ratio, grp.advantages.to(dev)[:, None], self.cfg.clip_eps_low,
                                           self.cfg.clip_eps_high)
            pg = pg + (per_tok * mask).sum()
            if self.cfg.kl_coef > 0:
                kl = kl + ((new - grp.ref_logprobs.to(dev)) * mask).sum()
            ntok += float(mask.sum())
        if ntok == 0:
            zero = sum(p.sum() for p in self.parameters()) * 0.0
            return zero, {**self._last_stats, "policy_loss": 0.0, "kl": 0.0, "entropy": 0.0, "tokens": 0.0}
        loss = (pg + self.cfg.kl_coef * kl - self.cfg.entropy_coef * ent) / ntok
        return loss, {**self._last_stats, "policy_loss": pg.detach() / ntok, "kl": kl.detach() / ntok,
                      "entropy": ent.detach() / ntok, "tokens": ntok}

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        n = min(8, len(self.prompts))
        passed, rsum = 0, 0.0
        for i in range(n):
            t = self.rollouts.rollout(self.prompts[i], self.tasks[i], group_size=1)[0]
            r = self.reward.score(t)
            rsum += r.value
            passed += int(bool(r.passed))
        return {"reward": rsum / max(n, 1), "pass_rate": passed / max(n, 1)}

    def state(self) -> Dict[str, Any]:
        return self.policy.state_for_checkpoint()

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.policy.load_checkpoint_state(state)

    def model_spec(self) -> Dict[str, Any]:
        return self.policy.spec.to_dict()

    def tokenizer_meta(self):
        return self.policy.tokenizer.metadata()
