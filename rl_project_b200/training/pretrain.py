"""Language-model pretraining (the algorithm, config and metric names of
``src/forgeline/training/pretrain.py``) on any token source: a corpus with ``sample_batch`` (memmap,
synthetic) or an iterator of ``(x, y)`` batches (streaming loaders, resident pools).

A corpus drawn onto a GPU is read one batch ahead: ``collect`` returns the batch staged during the
previous step and immediately stages the next one (its host-to-device copy is asynchronous, so it
overlaps the step about to run); checkpoints record the generator as it was before the staged draw.  Evaluation accumulates losses on the device and reads them back once per split.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable, Dict, List, Mapping, Optional, Tuple

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm

Batch = Tuple[torch.Tensor, torch.Tensor]


@dataclass
class PretrainConfig:
    batch_size: int = 16
    eval_batches: int = 20
    seed: int = 0


def _draw_fn(source: Any, batch_size: int, device: torch.device, gen: torch.Generator) -> Callable[[], Batch]:
    if hasattr(source, "sample_batch"):
        return lambda: source.sample_batch(batch_size, device, gen)

    def next_batch() -> Batch:
        x, y = next(source)
        return x.to(device, non_blocking=True), y.to(device, non_blocking=True)

    return next_batch


def _rows(batch: Batch, micro_step: int, n_micro: int) -> Batch:
    x, y = batch
    return (x[micro_step::n_micro], y[micro_step::n_micro]) if n_micro > 1 else (x, y)


class PretrainAlgorithm(PostTrainingAlgorithm):
    name = "pretrain"

    def __init__(self, model, train_corpus: Any, config: PretrainConfig, val_corpus: Optional[Any] = None,
                 device: torch.device | str = "cpu", tokenizer_meta: Optional[Dict[str, Any]] = None):
        block = getattr(train_corpus, "block_size", None)
        if block is not None and block != model.spec.block_size:
            raise ConfigError(f"corpus block_size {block} != model block_size {model.spec.block_size}")
        self.model, self.train, self.val, self.cfg = model, train_corpus, val_corpus, config
        self.spec = model.spec
        self.device = torch.device(device)
        self._tokenizer_meta = tokenizer_meta
        self.gen = torch.Generator().manual_seed(config.seed)
        self._draw = _draw_fn(train_corpus, config.batch_size, self.device, self.gen)
        # read-ahead for corpora drawn straight onto a GPU (their copy is asynchronous); other sources are read
        # when needed, so their cursors stay exact for checkpoints
        self._prefetch = hasattr(train_corpus, "sample_batch") and self.device.type == "cuda"
        self._staged: Optional[Batch] = None
        self._gen_before_stage = None
        self.tokens_seen = 0
        self.ema_loss: Optional[float] = None

    def parameters(self) -> List[nn.Parameter]:
        return [p for p in self.model.parameters() if p.requires_grad]

    def modules(self):
        return (self.model,)

    def collect(self, step: int) -> Batch:
        batch = self._staged if self._staged is not None else self._draw()
        self._staged = None
        if self._prefetch:
            self._gen_before_stage = self.gen.get_state()
            self._staged = self._draw()  # next step's batch is already on its way
        return batch

    def data_state(self) -> Dict[str, Any]:
        """Checkpointed data position: the generator as it was before the staged batch was drawn, so a
        resumed run draws that batch again."""
        st = super().data_state()
        if self._staged is not None:
            st["gen"] = ("torch_gen", self._gen_before_stage)
        return st

    def load_data_state(self, state: Mapping[str, Any]) -> None:
        super().load_data_state(state)
        self._staged = None

    def loss(self, batch: Batch, micro_step: int, n_micro: int):
        x, y = _rows(batch, micro_step, n_micro)
        _, loss = self.model(x, y)
        self.tokens_seen += x.numel()
        return loss, {"tokens_seen": float(self.tokens_seen)}

    def pipeline_inputs(self, batch: Batch, micro_step: int, n_micro: int) -> Batch:
        """``(input ids, targets)`` of one micro-batch, for pipeline-parallel schedules."""
        x, y = _rows(batch, micro_step, n_micro)
        self.tokens_seen += x.numel()
        return x, y

    def on_step_end(self, step: int, result) -> None:
        prev = self.ema_loss
        self.ema_loss = result.loss if prev is None else 0.95 * prev + 0.05 * result.loss
        result.metrics["ema_loss"] = self.ema_loss

    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        splits = {"train": self.train if hasattr(self.train, "sample_batch") else None, "val": self.val}
        out: Dict[str, float] = {}
        for name, corpus in splits.items():
            if corpus is None:
                continue
            draw = _draw_fn(corpus, self.cfg.batch_size, self.device, self.gen)
            total = torch.zeros((), device=self.device)
            for _ in range(self.cfg.eval_batches):
                total += self.model(*draw())[1].float()
            out[f"{name}_loss"] = float(total) / self.cfg.eval_batches
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
