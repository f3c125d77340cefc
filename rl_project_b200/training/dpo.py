"""Direct Preference Optimization (the objective and options of ``src/forgeline/training/dpo.py``)::

    z = beta * (log pi(y_w|x) - log pi_ref(y_w|x)) - beta * (log pi(y_l|x) - log pi_ref(y_l|x))
    L = (1 - eps) * softplus(-z) + eps * softplus(z)          (eps = label smoothing; softplus(-z) = -log sigmoid z)

with sequence scores reduced by ``sum`` or ``mean`` over response tokens, and ``reference_free`` dropping
the reference terms.

Execution plan of a step:

* ``collect`` draws the examples and scores them under the frozen reference right away -- the reference
  terms do not depend on the policy's weights, so they are computed once per step, outside the
  gradient-accumulation loop, and travel with the batch;
* each micro-batch scores chosen and rejected sides of all its examples in ONE policy forward: every
  ``prompt + response`` row is right-padded into a ``[2B, T]`` batch whose targets are -1 outside the
  response, and the fused LM-head log-prob kernel scores all rows at once.  Under causal attention the
  padding after a row cannot change its log-probs, so this equals scoring each example alone.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.training.common.logprobs import pack_prompt_response  # noqa: F401 - re-exported
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm


@dataclass
class DPOConfig:
    beta: float = 0.1
    batch_size: int = 4
    logprob_reduction: str = "sum"
    reference_free: bool = False
    label_smoothing: float = 0.0
    seed: int = 0

    def validate(self) -> None:
        if self.beta <= 0:
            raise ConfigError("DPO beta must be positive")
        if self.logprob_reduction not in ("sum", "mean"):
            raise ConfigError("logprob_reduction must be sum|mean")
        if not 0.0 <= self.label_smoothing < 0.5:
            raise ConfigError("label_smoothing must be in [0, 0.5)")


def dpo_loss(policy_chosen: torch.Tensor, policy_rejected: torch.Tensor, ref_chosen: torch.Tensor,
             ref_rejected: torch.Tensor, beta: float, label_smoothing: float = 0.0) -> Dict[str, torch.Tensor]:
    """Loss and implicit rewards from sequence log-probs ``[B]``."""
    implicit = beta * (torch.stack([policy_chosen, policy_rejected]) - torch.stack([ref_chosen, ref_rejected]))
    z = implicit[0] - implicit[1]
    per_pair = F.softplus(-z) if label_smoothing <= 0 else \
        (1.0 - label_smoothing) * F.softplus(-z) + label_smoothing * F.softplus(z)
    r = implicit.detach()
    return {"loss": per_pair.mean(), "chosen_reward": r[0], "rejected_reward": r[1], "margin": r[0] - r[1],
            "accuracy": (r[0] > r[1]).float()}


def sequence_logprobs(policy, pairs, reduction: str) -> torch.Tensor:
    """Per-row response log-prob, summed or averaged over the row's response tokens."""
    inputs, targets = pack_prompt_response(pairs, policy.pad_token_id)
    dev = policy.device
    targets = targets.to(dev)
    total = policy.token_logprobs(inputs.to(dev), targets).float().sum(1)
    return total if reduction == "sum" else total / (targets >= 0).sum(1).clamp(min=1)


@dataclass
class _Batch:
    examples: List[Dict[str, List[int]]]
    ref: torch.Tensor  # [2, B] reference scores (chosen, rejected); zeros when reference-free


class DPOAlgorithm(PostTrainingAlgorithm):
    name = "dpo"

    def __init__(self, policy, dataset, config: DPOConfig, eval_dataset=None):
        config.validate()
        if len(dataset) == 0:
            raise ConfigError("DPO dataset is empty")
        self.policy, self.dataset, self.eval_dataset, self.cfg = policy, dataset, eval_dataset, config
        self.rng = random.Random(config.seed)
        if not config.reference_free and not policy.has_adapter and policy.reference_model is None:
            policy.with_frozen_reference()

    # ------------------------------------------------------------ scoring
    def _both_sides(self, examples: Sequence[Dict[str, List[int]]]) -> torch.Tensor:
        """``[2, B]``: chosen and rejected scores of every example from one forward."""
        pairs = [(e["prompt"], e[side]) for side in ("chosen", "rejected") for e in examples]
        return sequence_logprobs(self.policy, pairs, self.cfg.logprob_reduction).view(2, len(examples))

    @torch.no_grad()
    def _reference(self, examples: Sequence[Dict[str, List[int]]]) -> torch.Tensor:
        if self.cfg.reference_free:
            return torch.zeros(2, len(examples), device=self.policy.device)
        with self.policy.reference():
            return self._both_sides(examples)

    # ------------------------------------------------------------ algorithm protocol
    def parameters(self) -> List[nn.Parameter]:
        return self.policy.trainable_parameters()

    def modules(self):
        return (self.policy.model,)

    def frozen_modules(self):
        return (self.policy.reference_model,) if self.policy.reference_model is not None else ()

    def collect(self, step: int) -> _Batch:
        examples = [self.dataset[self.rng.randrange(len(self.dataset))] for _ in range(self.cfg.batch_size)]
        return _Batch(examples, self._reference(examples))

    def loss(self, batch: _Batch, micro_step: int, n_micro: int):
        idx = list(range(micro_step, len(batch.examples), n_micro)) if n_micro > 1 else list(range(len(batch.examples)))
        if not idx:
            return torch.zeros((), device=self.policy.device, requires_grad=True), {}
        pol = self._both_sides([batch.examples[i] for i in idx])
        ref = batch.ref[:, idx]
        out = dpo_loss(pol[0], pol[1], ref[0], ref[1], self.cfg.beta, self.cfg.label_smoothing)
        return out["loss"], {"reward_margin": out["margin"].mean(), "chosen_reward": out["chosen_reward"].mean(),
                             "rejected_reward": out["rejected_reward"].mean(),
                             "preference_accuracy": out["accuracy"].mean()}

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        ds = self.eval_dataset or self.dataset
        examples = [ds[i] for i in range(min(len(ds), 32))]
        pol, ref = self._both_sides(examples), self._reference(examples)
        out = dpo_loss(pol[0], pol[1], ref[0], ref[1], self.cfg.beta)
        return {"loss": float(out["loss"]), "preference_accuracy": float(out["accuracy"].mean()),
                "reward_margin": float(out["margin"].mean())}

    def state(self) -> Dict[str, Any]:
        return self.policy.state_for_checkpoint()

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.policy.load_checkpoint_state(state)

    def model_spec(self) -> Dict[str, Any]:
        return self.policy.spec.to_dict()

    def tokenizer_meta(self):
        return self.policy.tokenizer.metadata()
