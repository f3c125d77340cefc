"""PPO for language-model policies (the options of ``src/forgeline/training/ppo.py``):

* ``ratio_level``: ``sequence_mean`` (ratio ``exp(mean_t(log pi - log pi_old))`` per sequence) or ``token``;
* ``kl_mode``: ``monitor`` (detached, logged), ``penalty`` (``kl_coef * KL`` added to the loss) or ``reward``
  (subtracted from the reward before the advantage);
* ``entropy_mode``: ``sampled_logprob`` (``-mean log pi(y_t)``) or ``full`` (exact entropy, from the fused
  LM-head kernel: no ``[B, T, V]`` logits);
* advantages ``reward - value`` (optionally normalised) and a value MSE loss.

Data flow: all prompts of a step are sampled together by the rollout engine; one scoring pass over the
left-padded batch yields old log-probs and values, one pass with adapters off / the frozen copy yields
the reference log-probs.  The surrogate (and penalty KL) run in the fused ``clipped_kl_loss`` op.

``ppo_epochs``: the objective averages ``ppo_epochs`` evaluations of the same loss at the same weights
(no optimizer step between them).  When the forward is deterministic (no active dropout) those
evaluations are identical, so the loss is evaluated once -- the same value and gradient for
``1 / ppo_epochs`` of the work; with dropout active each evaluation draws its own masks and all of them
run.
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
from rl_project_b200.ops.rl_loss import clipped_kl_loss
from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine
from rl_project_b200.rollouts.rewards.composite import score_trajectories
from rl_project_b200.training.common.advantages import normalize_advantages
from rl_project_b200.training.common.logprobs import kl_logprob_diff, masked_mean
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm

_CHOICES = {"ratio_level": ("sequence_mean", "token"), "kl_mode": ("monitor", "penalty", "reward"),
            "entropy_mode": ("sampled_logprob", "full")}


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
        for field_name, allowed in _CHOICES.items():
            if getattr(self, field_name) not in allowed:
                raise ConfigError(f"{field_name} must be {'|'.join(allowed)}")
        if not 0 < self.clip_ratio < 1:
            raise ConfigError("clip_ratio must be in (0, 1)")
        if min(self.ppo_epochs, self.prompts_per_step, self.samples_per_prompt) < 1:
            raise ConfigError("ppo_epochs, prompts_per_step and samples_per_prompt must be >= 1")


def ppo_clipped_objective(ratio: torch.Tensor, advantages: torch.Tensor, clip_ratio: float) -> torch.Tensor:
    """Elementwise ``-min(r A, clip(r, 1-eps, 1+eps) A)``."""
    return -torch.minimum(ratio * advantages, ratio.clamp(1.0 - clip_ratio, 1.0 + clip_ratio) * advantages)


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
    """``(prompts [N, P] left-padded, responses [N, R] right-padded, response mask [N, R] float)``."""
    from rl_project_b200.data.collators import pad_sequences

    prompts, _ = pad_sequences([t.prompt_ids.tolist() for t in trajectories], pad, "left")
    responses, mask = pad_sequences([t.response_ids.tolist() for t in trajectories], pad, "right")
    return prompts, responses, mask.float()


def _has_active_dropout(modules) -> bool:
    return any(isinstance(m, nn.Dropout) and m.p > 0 and m.training for mod in modules if mod is not None
               for m in mod.modules())


class PPOAlgorithm(PostTrainingAlgorithm):
    name = "ppo"

    def __init__(self, policy, prompts: Sequence[torch.Tensor], reward: RewardProvider, config: PPOConfig,
                 rollout: Optional[RolloutConfig] = None, tasks: Optional[Sequence[Dict[str, Any]]] = None):
        config.validate()
        if policy.value_head is None:
            raise ConfigError("PPO requires a policy with value_head=True")
        if not policy.has_adapter and policy.reference_model is None:
            policy.with_frozen_reference()
        self.policy, self.reward, self.cfg = policy, reward, config
        self.prompts = list(prompts)
        self.tasks = list(tasks) if tasks else [{} for _ in self.prompts]
        self.rollouts = RolloutEngine(policy, rollout or RolloutConfig(group_size=config.samples_per_prompt))
        self.rng = random.Random(config.seed)
        self._last_stats: Dict[str, float] = {}

    def parameters(self) -> List[nn.Parameter]:
        return self.policy.trainable_parameters()

    def modules(self):
        return (self.policy.model, self.policy.value_head)

    def frozen_modules(self):
        return (self.policy.reference_model,) if self.policy.reference_model is not None else ()

    # ------------------------------------------------------------ rollouts
    @torch.no_grad()
    def collect(self, step: int) -> PPOBatch:
        picks = [self.rng.randrange(len(self.prompts)) for _ in range(self.cfg.prompts_per_step)]
        groups = self.rollouts.rollout_many([self.prompts[i] for i in picks], [self.tasks[i] for i in picks],
                                            group_size=self.cfg.samples_per_prompt)
        trajs = [t for g in groups for t in g]
        rewards = torch.tensor(score_trajectories(self.reward, trajs), dtype=torch.float32)
        prompt, resp, mask = left_pad_batch(trajs, self.policy.pad_token_id)
        old_lp, old_v = self.policy.logprobs_and_values(prompt, resp)
        with self.policy.reference():
            ref_lp = self.policy.logprobs(prompt, resp)
        old_lp, ref_lp, old_v = old_lp.float().cpu(), ref_lp.float().cpu(), old_v.float().cpu()
        if self.cfg.kl_mode == "reward":
            rewards = rewards - self.cfg.kl_coef * kl_logprob_diff(ref_lp, old_lp, mask, clamp_min=None)
        self._last_stats = {"reward_mean": float(rewards.mean()),
                            "reward_std": float(rewards.std()) if len(trajs) > 1 else 0.0,
                            "response_len": float(mask.sum(1).mean())}
        return PPOBatch(prompt, resp, mask, old_lp, ref_lp, old_v, rewards, trajs)

    # ------------------------------------------------------------ objective
    def _terms(self, batch: PPOBatch, mask, returns, adv, old_lp, ref_lp) -> Dict[str, torch.Tensor]:
        """One evaluation of the PPO loss terms at the current weights."""
        cfg = self.cfg
        if cfg.entropy_mode == "full":
            new_lp, ent_tok = self.policy.logprobs_with_entropy(batch.prompt_ids, batch.response_ids)
            values = self.policy.values(batch.prompt_ids, batch.response_ids)
            entropy = masked_mean(ent_tok.float(), mask).mean()
        else:
            new_lp, values = self.policy.logprobs_and_values(batch.prompt_ids, batch.response_ids)
            entropy = -masked_mean(new_lp.float(), mask).mean()
        new_lp = new_lp.float()
        surrogate, _, _ = clipped_kl_loss(new_lp, old_lp, ref_lp, mask, adv, cfg.clip_ratio, 0.0, cfg.ratio_level,
                                          "logprob_diff_rows")
        kl = kl_logprob_diff(ref_lp, new_lp, mask).mean() if cfg.kl_mode == "penalty" else \
            masked_mean(old_lp - ref_lp, mask).mean().detach()
        value_loss = F.mse_loss(values.float(), returns)
        loss = surrogate + cfg.value_coef * value_loss - cfg.entropy_coef * entropy
        if cfg.kl_mode == "penalty":
            loss = loss + cfg.kl_coef * kl
        return {"loss": loss, "policy_loss": surrogate, "value_loss": value_loss, "kl": kl, "entropy": entropy}

    def loss(self, batch: PPOBatch, micro_step: int, n_micro: int):
        dev = self.policy.device
        mask, returns = batch.mask.to(dev), batch.rewards.to(dev)
        adv = returns - batch.old_values.to(dev)
        adv = (normalize_advantages(adv) if self.cfg.normalize_advantages else adv).detach()
        old_lp, ref_lp = batch.old_logprobs.to(dev), batch.ref_logprobs.to(dev)
        passes = self.cfg.ppo_epochs if _has_active_dropout(self.modules()) else 1
        runs = [self._terms(batch, mask, returns, adv, old_lp, ref_lp) for _ in range(passes)]
        mean = {k: sum(r[k] for r in runs) / passes for k in runs[0]}
        metrics: Dict[str, Any] = {k: v.detach() for k, v in mean.items() if k != "loss"}
        metrics.update(self._last_stats)
        metrics["advantage_mean"] = adv.mean()
        return mean["loss"], metrics

    def state(self) -> Dict[str, Any]:
        return self.policy.state_for_checkpoint()

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.policy.load_checkpoint_state(state)

    def model_spec(self) -> Dict[str, Any]:
        return self.policy.spec.to_dict()

    def tokenizer_meta(self):
        return self.policy.tokenizer.metadata()
