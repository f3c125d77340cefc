"""Language-model pretraining on a memmap / streaming / synthetic token source
(``src/forgeline/training/pretrain.py``)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm


@dataclass
class PretrainConfig:
    batch_size: int = 16
    eval_batches: int = 20
    seed: int = 0


class PretrainAlgorithm(PostTrainingAlgorithm):
    name = "pretrain"

    def __init__(self, model, train_corpus: Any, config: PretrainConfig, val_corpus: Optional[Any] = None,
                 device: torch.device | str = "cpu", tokenizer_meta: Optional[Dict[str, Any]] = None):
        self.model = model
        self.train = train_corpus
        self.val = val_corpus
        self.cfg = config
        self.device = torch.device(device)
        self._tokenizer_meta = tokenizer_meta
        self.gen = torch.Generator().manual_seed(config.seed)
        self.tokens_seen = 0
        self.ema_loss: Optional[float] = None
        self.spec = model.spec
        bs = getattr(train_corpus, "block_size", None)
        if bs is not None and bs != model.spec.block_size:
            raise ConfigError(f"corpus block_size {bs} != model block_size {model.spec.block_size}")

    def parameters(self) -> List[nn.Parameter]:
        return [p for p in self.model.parameters() if p.requires_grad]

    def modules(self):
        return (self.model,)

    def collect(self, step: int):
        if hasattr(self.train, "sample_batch"):
            return self.train.sample_batch(self.cfg.batch_size, self.device, self.gen)
        x, y = next(self.train)
        return x.to(self.device, non_blocking=True), y.to(self.device, non_blocking=True)

    def loss(self, batch, micro_step: int, n_micro: int):
        x, y = batch
        if n_micro > 1:
            x, y = x[micro_step::n_micro], y[micro_step::n_micro]
        _, loss = self.model(x, y)
        self.tokens_seen += int(x.numel())
        return loss, {"tokens_seen": float(self.tokens_seen)}

    def pipeline_inputs(self, batch, micro_step: int, n_micro: int):
        """``(input ids, targets)`` of one micro-batch, for pipeline-parallel schedules."""
        x, y = batch
        if n_micro > 1:
            x, y = x[micro_step::n_micro], y[micro_step::n_micro]
        self.tokens_seen += int(x.numel())
        return x, y

    def on_step_end(self, step: int, result) -> None:
        self.ema_loss = result.loss if self.ema_loss is None else 0.95 * self.ema_loss + 0.05 * result.loss
        result.metrics["ema_loss"] = self.ema_loss

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        out: Dict[str, float] = {}
        for name, corpus in (("train", self.train if hasattr(self.train, "sample_batch") else None), ("val", self.val)):
            if corpus is None:
                continue
            vals = []
            for _ in range(self.cfg.eval_batches):
                x, y = corpus.sample_batch(self.cfg.batch_size, self.device, self.gen)
                vals.append(float(self.model(x, y)[1]))
            out[f"{name}_loss"] = sum(vals) / len(vals)
        if "val_loss" in out:
            out["loss"] = out["val_loss"]
        return out

    def state(self) -> Dict[str, Any]:
        return {"model": self.model.state_dict()}

    def load_state(self, state: Mapping[str, Any]) -> None:
        from rl_project_b200.checkpoints.manager import load_model_state

        load_model_state(self.model, state["model"])

    def model_spec(self) -> Dict[str, Any]:
        return getattr(self.model, "module", self.model).spec.to_dict()

    def tokenizer_meta(self):
        return self._tokenizer_meta
