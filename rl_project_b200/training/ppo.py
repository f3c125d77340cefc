"""PPO for language-model policies (``src/forgeline/training/ppo.py`` switches:
``ratio_level`` sequence_mean | token, ``kl_mode`` monitor | penalty | reward,
``entropy_mode`` sampled_logprob | full; advantages ``reward - value``,
normalised, with a value MSE loss).

Rollouts of all prompts are sampled together and the old log-probs come from
the rollout itself (no second old-policy pass); ``entropy_mode="full"`` uses the
fused LM-head entropy kernel instead of materialising the logits.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.core.protocols import RewardProvider, Trajectory
from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine
from rl_project_b200.rollouts.rewards.composite import score_trajectories
from rl_project_b200.training.common.advantages import normalize_advantages
from rl_project_b200.ops.rl_loss import clipped_kl_loss
from rl_project_b200.training.common.logprobs import kl_logprob_diff, masked_mean
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm


@dataclass
class PPOConfig:
    prompts_per_step: int = 4
    samples_per_prompt: int = 1
    ppo_epochs: int = 3
    clip_ratio: float = 0.2
    value_coef: float = 0.5
    entropy_coef: float = 0.01
    kl_coef: float = 0.1
    ratio_level: str = "sequence_mean"
    kl_mode: str = "monitor"
    entropy_mode: str = "sampled_logprob"
    normalize_advantages: bool = True
    seed: int = 0

    def validate(self) -> None:
        if self.ratio_level not in ("sequence_mean", "token"):
            raise ConfigError("ratio_level must be sequence_mean|token")
        if self.kl_mode not in ("monitor", "penalty", "reward"):
            raise ConfigError("kl_mode must be monitor|penalty|reward")
        if self.entropy_mode not in ("sampled_logprob", "full"):
            raise ConfigError("entropy_mode must be sampled_logprob|full")
        if not 0 < self.clip_ratio < 1:
            raise ConfigError("clip_ratio must be in (0, 1)")
        if min(self.ppo_epochs, self.prompts_per_step, self.samples_per_prompt) < 1:
            raise ConfigError("ppo_epochs, prompts_per_step and samples_per_prompt must be >= 1")


def ppo_clipped_objective(ratio: torch.Tensor, advantages: torch.Tensor, clip_ratio: float) -> torch.Tensor:
    """Elementwise ``-min(r A, clip(r, 1-eps, 1+eps) A)``."""
    return -torch.min(ratio * advantages, torch.clamp(ratio, 1.0 - clip_ratio, 1.0 + clip_ratio) * advantages)


@dataclass
class PPOBatch:
    prompt_ids: torch.Tensor
    response_ids: torch.Tensor
    mask: torch.Tensor
    old_logprobs: torch.Tensor
    ref_logprobs: torch.Tensor
    old_values: torch.Tensor
    rewards: torch.Tensor
    trajectories: List[Trajectory]


def left_pad_batch(trajectories: Sequence[Trajectory], pad: int):
    P = max(t.prompt_ids.numel() for t in trajectories)
    R = max(t.response_length for t in trajectories)
    N = len(trajectories)
    prompt = torch.full((N, P), pad, dtype=torch.long)
    resp = torch.full((N, R), pad, dtype=torch.long)
    mask = torch.zeros((N, R))
    for i, t in enumerate(trajectories):
        prompt[i, P - t.prompt_ids.numel():] = t.prompt_ids
        resp[i, : t.response_length] = t.response_ids
        mask[i, : t.response_length] = 1.0
    return prompt, resp, mask


class PPOAlgorithm(PostTrainingAlgorithm):
    name = "ppo"

    def __init__(self, policy, prompts: Sequence[torch.Tensor], reward: RewardProvider, config: PPOConfig,
                 rollout: Optional[RolloutConfig] = None, tasks: Optional[Sequence[Dict[str, Any]]] = None):
        config.validate()
        if policy.value_head is None:
            raise ConfigError("PPO requires a policy with value_head=True")
        self.policy = policy
        if not policy.has_adapter and policy.reference_model is None:
            policy.with_frozen_reference()
        self.prompts = list(prompts)
        self.tasks = list(tasks) if tasks else [{} for _ in self.prompts]
        self.reward = reward
        self.cfg = config
        self.rollouts = RolloutEngine(policy, rollout or RolloutConfig(group_size=config.samples_per_prompt))
        self.rng = random.Random(config.seed)
        self._last_stats: Dict[str, float] = {}

    def parameters(self) -> List[nn.Parameter]:
        return self.policy.trainable_parameters()

    def modules(self):
        return (self.policy.model, self.policy.value_head)

    def frozen_modules(self):
        return (self.policy.reference_model,) if self.policy.reference_model is not None else ()

    @torch.no_grad()
    def collect(self, step: int) -> PPOBatch:
        idx = [self.rng.randrange(len(self.prompts)) for _ in range(self.cfg.prompts_per_step)]
        groups = self.rollouts.rollout_many([self.prompts[i] for i in idx], [self.tasks[i] for i in idx],
                                            group_size=self.cfg.samples_per_prompt)
        trajs = [t for g in groups for t in g]
        rewards = torch.tensor(score_trajectories(self.reward, trajs), dtype=torch.float32)
        prompt, resp, mask = left_pad_batch(trajs, self.policy.pad_token_id)
        old_lp, old_v = self.policy.logprobs_and_values(prompt, resp)
        with self.policy.reference():
            ref_lp = self.policy.logprobs(prompt, resp)
        old_lp, ref_lp = old_lp.float().cpu(), ref_lp.float().cpu()
        if self.cfg.kl_mode == "reward":
            rewards = rewards - self.cfg.kl_coef * kl_logprob_diff(ref_lp, old_lp, mask, clamp_min=None)
        self._last_stats = {"reward_mean": float(rewards.mean()),
                            "reward_std": float(rewards.std()) if len(trajs) > 1 else 0.0,
                            "response_len": float(mask.sum(1).mean())}
        return PPOBatch(prompt, resp, mask, old_lp, ref_lp, old_v.float().cpu(), rewards, trajs)

    def loss(self, batch: PPOBatch, micro_step: int, n_micro: int):
        dev = self.policy.device
        mask = batch.mask.to(dev)
        returns = batch.rewards.to(dev)
        adv = returns - batch.old_values.to(dev)
        if self.cfg.normalize_advantages:
            adv = normalize_advantages(adv)
        adv = adv.detach()
        old_lp, ref_lp = batch.old_logprobs.to(dev), batch.ref_logprobs.to(dev)
        total = torch.zeros((), device=dev)
        agg: Dict[str, torch.Tensor] = {}
        for _ in range(self.cfg.ppo_epochs):
            if self.cfg.entropy_mode == "full":
                new_lp, ent_tok = self.policy.logprobs_with_entropy(batch.prompt_ids, batch.response_ids)
                values = self.policy.values(batch.prompt_ids, batch.response_ids)
            else:
                new_lp, values = self.policy.logprobs_and_values(batch.prompt_ids, batch.response_ids)
                ent_tok = None
            new_lp = new_lp.float()
            # surrogate and (penalty mode) KL in one fused op; the KL penalty is added below
            pl, _, _ = clipped_kl_loss(new_lp, old_lp, ref_lp, mask, adv, self.cfg.clip_ratio, 0.0,
                                       self.cfg.ratio_level, "logprob_diff_rows")
            vl = F.mse_loss(values.float(), returns)
            if self.cfg.kl_mode == "penalty":
                kl = kl_logprob_diff(ref_lp, new_lp, mask).mean()
            else:
                kl = masked_mean(old_lp - ref_lp, mask).mean().detach()
            ent = masked_mean(ent_tok.float(), mask).mean() if ent_tok is not None else -masked_mean(new_lp, mask).mean()
            loss = pl + self.cfg.value_coef * vl - self.cfg.entropy_coef * ent
            if self.cfg.kl_mode == "penalty":
                loss = loss + self.cfg.kl_coef * kl
            total = total + loss
            for k, v in (("policy_loss", pl), ("value_loss", vl), ("kl", kl), ("entropy", ent)):
                agg[k] = agg.get(k, 0.0) + v.detach() / self.cfg.ppo_epochs
        metrics: Dict[str, Any] = dict(agg)
        metrics.update(self._last_stats)
        metrics["advantage_mean"] = adv.mean()
        return total / self.cfg.ppo_epochs, metrics

    def state(self) -> Dict[str, Any]:
        return self.policy.state_for_checkpoint()

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.policy.load_checkpoint_state(state)

    def model_spec(self) -> Dict[str, Any]:
        return self.policy.spec.to_dict()

    def tokenizer_meta(self):
        return self.policy.tokenizer.metadata()
