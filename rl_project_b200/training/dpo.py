"""Direct Preference Optimization (``src/forgeline/training/dpo.py`` objective):

    L = -log sigmoid( beta (log pi(y_w|x) - log pi_ref(y_w|x)) - beta (log pi(y_l|x) - log pi_ref(y_l|x)) )

with ``logprob_reduction`` sum | mean, ``reference_free`` and label smoothing.

Batched: every (prompt + chosen) and (prompt + rejected) sequence of the
micro-batch is right-padded into ONE forward pass.  With causal attention,
padding placed after a sequence cannot change its log-probs, and every row
keeps positions 0..L-1, so this equals the reference's one-forward-per-example
loop exactly while running one fused LM-head kernel for the whole batch.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.errors import ConfigError
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
    cr = beta * (policy_chosen - ref_chosen)
    rr = beta * (policy_rejected - ref_rejected)
    z = cr - rr
    loss = -F.logsigmoid(z) * (1 - label_smoothing) - F.logsigmoid(-z) * label_smoothing if label_smoothing > 0 \
        else -F.logsigmoid(z)
    return {"loss": loss.mean(), "chosen_reward": cr.detach(), "rejected_reward": rr.detach(),
            "margin": (cr - rr).detach(), "accuracy": (cr > rr).float().detach()}


def pack_prompt_response(pairs: Sequence[Tuple[List[int], List[int]]], pad: int):
    """Right-padded ``inputs [B, T]`` and ``targets [B, T]`` (-1 outside each response)."""
    seqs = [list(p) + list(r) for p, r in pairs]
    T = max(len(s) for s in seqs) - 1
    inputs = torch.full((len(seqs), T), pad, dtype=torch.long)
    targets = torch.full((len(seqs), T), -1, dtype=torch.long)
    for i, ((p, r), s) in enumerate(zip(pairs, seqs)):
        L = len(s)
        inputs[i, : L - 1] = torch.tensor(s[:-1])
        targets[i, len(p) - 1: L - 1] = torch.tensor(s[len(p):])
    return inputs, targets


def sequence_logprobs(policy, pairs, reduction: str) -> torch.Tensor:
    inputs, targets = pack_prompt_response(pairs, policy.pad_token_id)
    dev = policy.device
    targets = targets.to(dev)
    lp = policy.token_logprobs(inputs.to(dev), targets).float()
    if reduction == "sum":
        return lp.sum(1)
    return lp.sum(1) / (targets >= 0).sum(1).clamp(min=1)


class DPOAlgorithm(PostTrainingAlgorithm):
    name = "dpo"

    def __init__(self, policy, dataset, config: DPOConfig, eval_dataset=None):
        config.validate()
        self.policy = policy
        self.dataset = dataset
        self.eval_dataset = eval_dataset
        self.cfg = config
        self.rng = random.Random(config.seed)
        if not config.reference_free and not policy.has_adapter and policy.reference_model is None:
            policy.with_frozen_reference()
        if len(dataset) == 0:
            raise ConfigError("DPO dataset is empty")

    def parameters(self) -> List[nn.Parameter]:
        return self.policy.trainable_parameters()

    def modules(self):
        return (self.policy.model,)

    def frozen_modules(self):
        return (self.policy.reference_model,) if self.policy.reference_model is not None else ()

    def collect(self, step: int):
        return [self.dataset[self.rng.randrange(len(self.dataset))] for _ in range(self.cfg.batch_size)]

    def _scores(self, examples) -> Tuple[torch.Tensor, torch.Tensor]:
        pairs = [(e["prompt"], e["chosen"]) for e in examples] + [(e["prompt"], e["rejected"]) for e in examples]
        s = sequence_logprobs(self.policy, pairs, self.cfg.logprob_reduction)
        n = len(examples)
        return s[:n], s[n:]

    def loss(self, batch, micro_step: int, n_micro: int):
        chunk = batch[micro_step::n_micro] if n_micro > 1 else batch
        if not chunk:
            return torch.zeros((), device=self.policy.device, requires_grad=True), {}
        pc, pr = self._scores(chunk)
        if self.cfg.reference_free:
            rc, rr = torch.zeros_like(pc), torch.zeros_like(pr)
        else:
            with torch.no_grad(), self.policy.reference():
                rc, rr = self._scores(chunk)
        out = dpo_loss(pc, pr, rc, rr, self.cfg.beta, self.cfg.label_smoothing)
        return out["loss"], {"reward_margin": out["margin"].mean(), "chosen_reward": out["chosen_reward"].mean(),
                             "rejected_reward": out["rejected_reward"].mean(),
                             "preference_accuracy": out["accuracy"].mean()}

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        ds = self.eval_dataset or self.dataset
        ex = [ds[i] for i in range(min(len(ds), 32))]
        pc, pr = self._scores(ex)
        if self.cfg.reference_free:
            rc, rr = torch.zeros_like(pc), torch.zeros_like(pr)
        else:
            with self.policy.reference():
                rc, rr = self._scores(ex)
        out = dpo_loss(pc, pr, rc, rr, self.cfg.beta)
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
