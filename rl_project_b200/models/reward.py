"""Reward models (contract of ``src/forgeline/models/reward.py``: class names, constructor arguments, the
``reward_head`` parameter name and the ``{model, pooling}`` checkpoint dict).

``SequenceRewardModel`` pools the backbone's final hidden states with one weighted reduction: a ``[B, T]``
pooling matrix (a one-hot at each row's last real token for ``last``, ``mask / length`` for ``mean``)
contracted with ``h [B, T, C]``, followed by the bias-free scalar head -- the same code path with or
without an attention mask (no mask = every position is real).

``EncoderRewardModel`` is the text-level variant on a HuggingFace encoder (its CLS state through a small
MLP head): ``regression`` (sigmoid output, MSE to scalar targets) or ``preference`` (raw score,
Bradley-Terry on chosen / rejected texts).  Both fits run through one epoch loop over index batches.
"""

from __future__ import annotations

from typing import Any, Callable, Dict, Iterable, List, Mapping, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.core.errors import ConfigError, OptionalDependencyError
from rl_project_b200.models.transformer.model import TransformerLM


def pooling_weights(mask: torch.Tensor, pooling: str) -> torch.Tensor:
    """``[B, T]`` weights that reduce hidden states to one vector per row."""
    m = mask.float()
    if pooling == "mean":
        return m / m.sum(1, keepdim=True).clamp_min(1.0)
    last = (m.sum(1).long() - 1).clamp_min(0)
    return F.one_hot(last, m.shape[1]).float()


class SequenceRewardModel(nn.Module):
    def __init__(self, spec: ModelSpec, backbone: Optional[TransformerLM] = None, pooling: str = "last"):
        super().__init__()
        if pooling not in ("last", "mean"):
            raise ValueError("pooling must be 'last' or 'mean'")
        self.spec, self.pooling = spec, pooling
        self.backbone = backbone if backbone is not None else TransformerLM(spec)
        self.reward_head = nn.Linear(spec.n_embd, 1, bias=False)

    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        h = self.backbone.forward_hidden(input_ids)
        mask = attention_mask if attention_mask is not None else torch.ones(h.shape[:2], device=h.device)
        w = pooling_weights(mask.to(h.device), self.pooling).to(h.dtype)
        pooled = torch.bmm(w.unsqueeze(1), h).squeeze(1)
        return self.reward_head(pooled.to(self.reward_head.weight.dtype)).squeeze(-1)

    def freeze_backbone(self) -> None:
        self.backbone.requires_grad_(False)

    def state_for_checkpoint(self) -> Dict[str, Any]:
        return {"model": self.state_dict(), "pooling": self.pooling}

    def load_checkpoint_state(self, state: Mapping[str, Any]) -> None:
        self.load_state_dict(state["model"])


def bradley_terry_loss(chosen_scores: torch.Tensor, rejected_scores: torch.Tensor) -> torch.Tensor:
    """Mean ``-log sigmoid(chosen - rejected)`` (computed in fp32)."""
    return F.softplus(rejected_scores.float() - chosen_scores.float()).mean()


class EncoderRewardModel(nn.Module):
    """Encoder reward model on raw text; head: dropout, ``h -> h/2`` GELU layer, then a scalar read-out
    (``regression`` adds dropout before it and a sigmoid after it)."""

    _OBJECTIVES = ("regression", "preference")

    def __init__(self, backbone: str = "bert-base-uncased", objective: str = "regression", dropout: float = 0.1,
                 max_length: int = 128):
        super().__init__()
        if objective not in self._OBJECTIVES:
            raise ConfigError("objective must be regression|preference")
        try:
            from transformers import AutoModel, AutoTokenizer
        except ImportError as exc:
            raise OptionalDependencyError("transformers is not installed", hint="pip install transformers") from exc
        self.objective, self.max_length = objective, max_length
        self.tokenizer = AutoTokenizer.from_pretrained(backbone)
        self.encoder = AutoModel.from_pretrained(backbone)
        self.head = self._head(self.encoder.config.hidden_size, dropout, objective == "regression")
        self.trained = False

    @staticmethod
    def _head(h: int, dropout: float, bounded: bool) -> nn.Sequential:
        readout = [nn.Dropout(dropout), nn.Linear(h // 2, 1), nn.Sigmoid()] if bounded else [nn.Linear(h // 2, 1)]
        return nn.Sequential(nn.Dropout(dropout), nn.Linear(h, h // 2), nn.GELU(), *readout)

    def forward(self, texts: Iterable[str]) -> torch.Tensor:
        dev = next(self.parameters()).device
        enc = self.tokenizer(list(texts), return_tensors="pt", padding=True, truncation=True,
                             max_length=self.max_length).to(dev)
        cls = self.encoder(input_ids=enc["input_ids"], attention_mask=enc["attention_mask"]).last_hidden_state[:, 0]
        return self.head(cls).squeeze(-1)

    @torch.no_grad()
    def score_texts(self, texts: Iterable[str], probability: bool = True) -> torch.Tensor:
        self.eval()
        s = self(texts)
        return s.sigmoid() if probability and self.objective == "preference" else s

    def _epochs(self, n: int, batch_size: int, epochs: int, opt: torch.optim.Optimizer,
                loss_of: Callable[[List[int]], torch.Tensor], order: Callable[[], List[int]],
                clip: Optional[float] = None) -> List[float]:
        """Mean loss per epoch; each epoch visits ``order()`` in ``batch_size`` slices."""
        history = []
        self.train()
        for _ in range(epochs):
            idx = order()
            losses = []
            for lo in range(0, n, batch_size):
                loss = loss_of(idx[lo:lo + batch_size])
                opt.zero_grad()
                loss.backward()
                if clip:
                    nn.utils.clip_grad_norm_(self.parameters(), clip)
                opt.step()
                losses.append(float(loss.detach()))
            history.append(sum(losses) / max(len(losses), 1))
        self.trained = True
        return history

    def fit_regression(self, texts: Sequence[str], targets: Iterable[float], epochs: int = 3, lr: float = 1e-4,
                       batch_size: int = 16) -> List[float]:
        y = torch.tensor(list(targets), dtype=torch.float32)

        def loss_of(idx):
            pred = self([texts[i] for i in idx])
            return F.mse_loss(pred, y[idx].to(pred.device))

        return self._epochs(len(texts), batch_size, epochs, torch.optim.Adam(self.parameters(), lr=lr), loss_of,
                            lambda: list(range(len(texts))))

    def fit_preference(self, pairs: Sequence[Sequence[str]], epochs: int = 3, lr: float = 2e-5, batch_size: int = 16,
                       seed: int = 0) -> List[float]:
        gen = torch.Generator().manual_seed(seed)

        def loss_of(idx):
            return bradley_terry_loss(self([pairs[j][0] for j in idx]), self([pairs[j][1] for j in idx]))

        return self._epochs(len(pairs), batch_size, epochs, torch.optim.AdamW(self.parameters(), lr=lr), loss_of,
                            lambda: torch.randperm(len(pairs), generator=gen).tolist(), clip=1.0)
