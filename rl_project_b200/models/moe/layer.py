"""Mixture-of-experts layer with sort-based dispatch.

The reference loops ``topk x n_experts`` with boolean masks
(``src/forgeline/models/moe/layer.py:32-38``).  Here the (token, slot) pairs
are sorted by expert once, each expert runs on its contiguous segment, and
the weighted outputs are scattered back with one ``index_add_``.  The same
permutation feeds the expert-parallel all-to-all (parallel/expert.py).
Parameter names (``gate``, ``experts.{e}.w*``, ``shared_experts.w*``) match
the reference checkpoints.
"""

from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn as nn

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.models.moe.gate import ExpertGate
from rl_project_b200.models.transformer.feedforward import make_ffn


def sort_by_expert(indices: torch.Tensor, n_experts: int):
    """``indices [N, k]`` -> (order, token_of_slot, counts[E]) with slots grouped by expert."""
    flat = indices.reshape(-1)
    order = torch.sort(flat, stable=True).indices
    counts = torch.bincount(flat, minlength=n_experts)
    return order, order // indices.shape[1], counts


class MoELayer(nn.Module):
    def __init__(self, spec: ModelSpec):
        super().__init__()
        self.n_experts = spec.n_experts
        self.n_experts_active = spec.n_experts_active
        self.n_shared_experts = spec.n_shared_experts
        self.gate = ExpertGate(spec)
        hidden = spec.expert_hidden
        self.experts = nn.ModuleList([make_ffn(spec, hidden) for _ in range(spec.n_experts)])
        # the reference builds ONE shared FFN whatever n_shared_experts says; its
        # width here is n_shared * expert width, which equals it when n_shared == 1
        self.shared_experts = (make_ffn(spec, hidden * max(1, spec.n_shared_experts) if spec.moe_d_ff else None)
                               if spec.n_shared_experts > 0 else None)
        self.expert_group = None  # set by the expert-parallel strategy
        self.local_experts = list(range(spec.n_experts))

    @property
    def aux_loss(self):
        return self.gate.aux_loss

    def run_experts(self, xs: torch.Tensor, counts: List[int], first_expert: int = 0) -> torch.Tensor:
        outs = []
        start = 0
        for j, c in enumerate(counts):
            if c:
                outs.append(self.experts[first_expert + j](xs[start:start + c]))
            start += c
        if not outs:
            return xs.new_zeros(xs.shape)
        return torch.cat(outs, 0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, C = x.shape
        xf = x.reshape(-1, C)
        weights, indices = self.gate(xf)
        if self.expert_group is not None:
            from rl_project_b200.parallel.expert import expert_parallel_moe

            y = expert_parallel_moe(self, xf, weights, indices)
        else:
            order, tok, counts = sort_by_expert(indices, self.n_experts)
            xs = xf.index_select(0, tok)
            ys = self.run_experts(xs, counts.tolist())
            w = weights.reshape(-1).index_select(0, order).unsqueeze(-1).to(ys.dtype)
            y = torch.zeros_like(xf).index_add_(0, tok, ys * w)
        if self.shared_experts is not None:
            y = y + self.shared_experts(xf)
        return y.view(B, T, C)
