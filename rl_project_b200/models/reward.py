"""Reward models (``src/forgeline/models/reward.py`` contract): a native
transformer backbone with a scalar head (last or mean pooling), the
Bradley-Terry pairwise loss, and an optional HuggingFace encoder reward model."""

from __future__ import annotations

import random
from typing import Any, Dict, Mapping, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.core.errors import ConfigError, OptionalDependencyError
from rl_project_b200.models.transformer.model import TransformerLM


class SequenceRewardModel(nn.Module):
    def __init__(self, spec: ModelSpec, backbone: Optional[TransformerLM] = None, pooling: str = "last"):
        super().__init__()
        if pooling not in ("last", "mean"):
            raise ValueError("pooling must be 'last' or 'mean'")
        self.spec = spec
        self.pooling = pooling
        self.backbone = backbone or TransformerLM(spec)
        self.reward_head = nn.Linear(spec.n_embd, 1, bias=False)

    def forward(self, input_ids: torch.Tensor, attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        h = self.backbone.forward_hidden(input_ids)
        if self.pooling == "mean":
            if attention_mask is None:
                pooled = h.mean(1)
            else:
                m = attention_mask.unsqueeze(-1).to(h.dtype)
                pooled = (h * m).sum(1) / m.sum(1).clamp(min=1.0)
        elif attention_mask is None:
            pooled = h[:, -1]
        else:
            last = attention_mask.long().sum(1).clamp(min=1) - 1
            pooled = h[torch.arange(h.shape[0], device=h.device), last]
        return self.reward_head(pooled.to(self.reward_head.weight.dtype)).squeeze(-1)

    def freeze_backbone(self) -> None:
        for p in self.backbone.parameters():
            p.requires_grad = False

    def state_for_checkpoint(self) -> Dict[str, Any]:
        return {"model": self.state_dict(), "pooling": self.pooling}

    def load_checkpoint_state(self, state: Mapping[str, Any]) -> None:
        self.load_state_dict(state["model"])


def bradley_terry_loss(chosen_scores: torch.Tensor, rejected_scores: torch.Tensor) -> torch.Tensor:
    return -F.logsigmoid(chosen_scores.float() - rejected_scores.float()).mean()


class EncoderRewardModel(nn.Module):
    """Encoder (CLS) reward model on text, ``regression`` (sigmoid + MSE) or ``preference`` (Bradley-Terry)."""

    def __init__(self, backbone: str = "bert-base-uncased", objective: str = "regression", dropout: float = 0.1,
                 max_length: int = 128):
        super().__init__()
        if objective not in ("regression", "preference"):
            raise ConfigError("objective must be regression|preference")
        try:
            from transformers import AutoModel, AutoTokenizer
        except ImportError as exc:
            raise OptionalDependencyError("transformers is not installed", hint="pip install transformers") from exc
        self.objective, self.max_length = objective, max_length
        self.tokenizer = AutoTokenizer.from_pretrained(backbone)
        self.encoder = AutoModel.from_pretrained(backbone)
        h = self.encoder.config.hidden_size
        layers = [nn.Dropout(dropout), nn.Linear(h, h // 2), nn.GELU()]
        layers += [nn.Dropout(dropout), nn.Linear(h // 2, 1), nn.Sigmoid()] if objective == "regression" \
            else [nn.Linear(h // 2, 1)]
        self.head = nn.Sequential(*layers)
        self.trained = False

    def forward(self, texts) -> torch.Tensor:
        enc = self.tokenizer(list(texts), return_tensors="pt", padding=True, truncation=True, max_length=self.max_length)
        dev = next(self.parameters()).device
        out = self.encoder(input_ids=enc["input_ids"].to(dev), attention_mask=enc["attention_mask"].to(dev))
        return self.head(out.last_hidden_state[:, 0]).squeeze(-1)

    @torch.no_grad()
    def score_texts(self, texts, probability: bool = True) -> torch.Tensor:
        self.eval()
        s = self(texts)
        return torch.sigmoid(s) if (probability and self.objective == "preference") else s

    def _fit(self, batches, loss_fn, epochs, opt, clip=None) -> list:
        hist = []
        self.train()
        for _ in range(epochs):
            tot, n = 0.0, 0
            for b in batches():
                loss = loss_fn(b)
                opt.zero_grad()
                loss.backward()
                if clip:
                    torch.nn.utils.clip_grad_norm_(self.parameters(), clip)
                opt.step()
                tot += float(loss.detach())
                n += 1
            hist.append(tot / max(n, 1))
        self.trained = True
        return hist

    def fit_regression(self, texts, targets, epochs: int = 3, lr: float = 1e-4, batch_size: int = 16) -> list:
        y = torch.tensor(list(targets), dtype=torch.float32)
        opt = torch.optim.Adam(self.parameters(), lr=lr)

        def batches():
            for i in range(0, len(texts), batch_size):
                yield i

        def loss_fn(i):
            p = self(texts[i:i + batch_size])
            return F.mse_loss(p, y[i:i + batch_size].to(p.device))

        return self._fit(batches, loss_fn, epochs, opt)

    def fit_preference(self, pairs, epochs: int = 3, lr: float = 2e-5, batch_size: int = 16, seed: int = 0) -> list:
        opt = torch.optim.AdamW(self.parameters(), lr=lr)
        rng = random.Random(seed)

        def batches():
            order = list(range(len(pairs)))
            rng.shuffle(order)
            for i in range(0, len(order), batch_size):
                yield order[i:i + batch_size]

        def loss_fn(idx):
            return bradley_terry_loss(self([pairs[j][0] for j in idx]), self([pairs[j][1] for j in idx]))

        return self._fit(batches, loss_fn, epochs, opt, clip=1.0)
