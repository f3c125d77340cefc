"""Supervised fine-tuning with prompt masking (``src/forgeline/training/sft.py``).

Token-mean cross-entropy over response tokens, computed by the fused LM-head
log-softmax kernel.  The data side is either a ``SupervisedDataset`` of
(prompt, response) records (shuffled epochs, seeded) or any object with
``next_batch() -> SupervisedBatch`` (e.g. ``data.synthetic.SyntheticSFTSource``);
host batches are copied to the device with ``non_blocking`` from pinned memory.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.data.collators import IGNORE_INDEX, SupervisedBatch, collate_supervised
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm


@dataclass
class SFTConfig:
    batch_size: int = 8
    max_length: int = 256
    mask_prompt: bool = True
    seed: int = 0


class SFTAlgorithm(PostTrainingAlgorithm):
    name = "sft"

    def __init__(self, policy, dataset: Any, config: SFTConfig, eval_dataset: Optional[Any] = None):
        self.policy = policy
        self.dataset = dataset
        self.eval_dataset = eval_dataset
        self.cfg = config
        self.streaming = hasattr(dataset, "next_batch")
        if not self.streaming and len(dataset) == 0:
            raise ConfigError("SFT dataset is empty")
        self.rng = random.Random(config.seed)
        self._order: List[int] = []

    def parameters(self) -> List[nn.Parameter]:
        return self.policy.trainable_parameters()

    def modules(self):
        return (self.policy.model,)

    def frozen_modules(self):
        return (self.policy.reference_model,) if getattr(self.policy, "reference_model", None) is not None else ()

    def _indices(self, n: int) -> List[int]:
        out = []
        while len(out) < n:
            if not self._order:
                self._order = list(range(len(self.dataset)))
                self.rng.shuffle(self._order)
            out.append(self._order.pop())
        return out

    def _collate(self, examples) -> SupervisedBatch:
        return collate_supervised(examples, pad_value=self.policy.pad_token_id,
                                  max_length=min(self.cfg.max_length, self.policy.max_length + 1),
                                  mask_prompt=self.cfg.mask_prompt)

    def collect(self, step: int) -> SupervisedBatch:
        if self.streaming:
            batch = self.dataset.next_batch()
        else:
            batch = self._collate([self.dataset[i] for i in self._indices(self.cfg.batch_size)])
        return batch.to(self.policy.device, non_blocking=True)

    def _ce(self, batch: SupervisedBatch) -> torch.Tensor:
        return self.policy.token_ce(batch.input_ids, batch.targets)

    def loss(self, batch: SupervisedBatch, micro_step: int, n_micro: int):
        if n_micro > 1:
            batch = batch.micro(micro_step, n_micro)
        loss = self._ce(batch)
        return loss, {"response_tokens": (batch.targets != IGNORE_INDEX).sum()}

    def pipeline_inputs(self, batch: SupervisedBatch, micro_step: int, n_micro: int):
        """``(input ids, targets)`` of one micro-batch, for pipeline-parallel schedules."""
        if n_micro > 1:
            batch = batch.micro(micro_step, n_micro)
        return batch.input_ids, batch.targets

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        ds = self.eval_dataset or self.dataset
        if hasattr(ds, "next_batch"):
            return {"loss": float(self._ce(ds.next_batch().to(self.policy.device)))}
        n = min(len(ds), 4 * self.cfg.batch_size)
        losses = [float(self._ce(self._collate([ds[j] for j in range(i, min(i + self.cfg.batch_size, n))])
                                 .to(self.policy.device)))
                  for i in range(0, n, self.cfg.batch_size)]
        return {"loss": sum(losses) / max(1, len(losses))}

    def state(self) -> Dict[str, Any]:
        return self.policy.state_for_checkpoint()

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.policy.load_checkpoint_state(state)

    def model_spec(self) -> Dict[str, Any]:
        return self.policy.spec.to_dict()

    def tokenizer_meta(self):
        tok = getattr(self.policy, "tokenizer", None)
        return tok.metadata() if tok is not None and hasattr(tok, "metadata") else None
