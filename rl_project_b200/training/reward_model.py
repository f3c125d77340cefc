"""Reward-model training: a scalar head on the policy backbone fitted to preference pairs with the
Bradley-Terry objective ``-log sigmoid(r_chosen - r_rejected)`` (reference:
``src/forgeline/training/reward_model.py``).

Each step scores the chosen and the rejected completions of a batch in ONE forward pass: the 2B
sequences (prompt + response, cut to their last ``max_length`` tokens) are padded into a single batch,
so the backbone runs once per micro-batch rather than twice.  Batches are drawn without replacement, a
seeded shuffle per epoch.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.data.collators import pad_sequences
from rl_project_b200.models.reward import bradley_terry_loss
from rl_project_b200.training.common.sampling import EpochSampler
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm


@dataclass
class RewardModelConfig:
    batch_size: int = 8
    freeze_backbone: bool = False
    max_length: int = 256
    seed: int = 0


class RewardModelAlgorithm(PostTrainingAlgorithm):
    name = "reward_model"

    def __init__(self, model, dataset, config: RewardModelConfig, eval_dataset=None, pad_token_id: int = 0,
                 tokenizer_meta: Optional[Dict[str, Any]] = None):
        if len(dataset) == 0:
            raise ConfigError("reward-model dataset is empty")
        self.model = model
        self.dataset = dataset
        self.eval_dataset = eval_dataset
        self.cfg = config
        self.pad = pad_token_id
        self._tok_meta = tokenizer_meta
        self.sampler = EpochSampler(len(dataset), config.seed)
        if config.freeze_backbone:
            model.freeze_backbone()

    # ------------------------------------------------------------ trainer hooks
    def parameters(self) -> List[nn.Parameter]:
        return [p for p in self.model.parameters() if p.requires_grad]

    def modules(self):
        return (self.model,)

    def collect(self, step: int):
        return [self.dataset[i] for i in self.sampler.take(self.cfg.batch_size)]

    def _pair_scores(self, examples: Sequence[Mapping[str, List[int]]]) -> Tuple[torch.Tensor, torch.Tensor]:
        """(chosen scores, rejected scores) from one forward over both sides of every pair."""
        keep = self.cfg.max_length
        seqs = [(e["prompt"] + e[side])[-keep:] for side in ("chosen", "rejected") for e in examples]
        ids, mask = pad_sequences(seqs, self.pad, "right")
        dev = next(self.model.parameters()).device
        scores = self.model(ids.to(dev), mask.to(dev)).float()
        return scores[:len(examples)], scores[len(examples):]

    def loss(self, batch, micro_step: int, n_micro: int):
        part = batch if n_micro <= 1 else batch[micro_step::n_micro]
        chosen, rejected = self._pair_scores(part)
        gap = chosen - rejected
        return bradley_terry_loss(chosen, rejected), {"accuracy": (gap > 0).float().mean(),
                                                      "margin": gap.detach().mean()}

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        ds = self.eval_dataset if self.eval_dataset is not None else self.dataset
        chosen, rejected = self._pair_scores([ds[i] for i in range(min(len(ds), 32))])
        return {"loss": float(bradley_terry_loss(chosen, rejected)), "accuracy": float((chosen > rejected).float().mean())}

    # ------------------------------------------------------------ checkpoint contract
    def state(self) -> Dict[str, Any]:
        return self.model.state_for_checkpoint()

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.model.load_checkpoint_state(state)

    def model_spec(self) -> Dict[str, Any]:
        return self.model.spec.to_dict()

    def tokenizer_meta(self):
        return self._tok_meta
