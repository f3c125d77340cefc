"""Expert router (``src/forgeline/models/moe/gate.py:15-79`` semantics).

Scores = softmax or sigmoid of ``x W^T`` in fp32; the aux-loss-free bias
(``expert_bias``) only affects which experts are selected, never the weights;
group-limited routing keeps the top ``n_limited_groups`` groups by their max
score; sigmoid weights are renormalised; ``route_scale`` multiplies the
result.  In training the bias moves by ``bias_update_speed * (mean - count)``
(aux-free) or a Switch-style load-balance loss is produced.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.config import ModelSpec


class ExpertGate(nn.Module):
    def __init__(self, spec: ModelSpec):
        super().__init__()
        self.dim = spec.n_embd
        self.topk = spec.n_experts_active
        self.n_experts = spec.n_experts
        self.score_func = spec.score_func
        self.route_scale = spec.route_scale
        self.aux_loss_free = spec.aux_loss_free
        self.bias_update_speed = spec.bias_update_speed
        self.aux_loss_weight = spec.moe_aux_loss_weight
        self.n_expert_groups = spec.n_expert_groups
        self.n_limited_groups = spec.n_limited_groups
        self.weight = nn.Parameter(torch.empty(spec.n_experts, spec.n_embd))
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.aux_loss_free:
            self.register_buffer("expert_bias", torch.zeros(spec.n_experts, dtype=torch.float32))
        self._aux_loss: Optional[torch.Tensor] = None
        self.last_counts: Optional[torch.Tensor] = None
        self.count_group = None  # data-parallel group: bias updates then use global counts (identical on all ranks)

    @property
    def aux_loss(self) -> Optional[torch.Tensor]:
        return self._aux_loss

    def _fused_ok(self, x: torch.Tensor) -> bool:
        from rl_project_b200.ops._ext import available

        return (x.is_cuda and available() and self.n_experts <= 256 and self.topk <= 16
                and self.n_expert_groups <= 32 and self.n_experts % self.n_expert_groups == 0)

    def route(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Return ``(weights [N,k] fp32, indices [N,k], scores [N,E] fp32)``.  On CUDA everything after the
        router GEMM is one kernel (csrc/moe_router.cu); its counts are kept for ``forward``."""
        if self._fused_ok(x):
            logits = F.linear(x.float(), self.weight.float())
            bias = self.expert_bias.float() if self.aux_loss_free else None  # the buffer follows .to(dtype)
            w, idx, scores, counts = _FusedRoute.apply(
                logits, bias, self.topk, self.n_expert_groups,
                self.n_limited_groups, self.score_func == "sigmoid", float(self.route_scale))
            self._fused_counts = counts
            return w, idx, scores
        self._fused_counts = None
        scores = F.linear(x.float(), self.weight.float())
        scores = scores.softmax(-1) if self.score_func == "softmax" else scores.sigmoid()
        select = scores + self.expert_bias if self.aux_loss_free else scores
        if 1 < self.n_expert_groups and self.n_limited_groups < self.n_expert_groups:
            N = x.shape[0]
            g = select.view(N, self.n_expert_groups, -1)
            keep = g.amax(-1).topk(self.n_limited_groups, dim=-1).indices
            gmask = torch.zeros(N, self.n_expert_groups, dtype=torch.bool, device=x.device)
            gmask.scatter_(1, keep, True)
            select = select.masked_fill(~gmask.repeat_interleave(self.n_experts // self.n_expert_groups, 1),
                                        float("-inf"))
        idx = select.topk(self.topk, dim=-1).indices
        w = scores.gather(1, idx)
        if self.score_func == "sigmoid":
            w = w / (w.sum(-1, keepdim=True) + 1e-8)
        return w * self.route_scale, idx, scores

    def forward(self, x: torch.Tensor):
        w, idx, scores = self.route(x)
        fc = getattr(self, "_fused_counts", None)
        counts = fc.float() if fc is not None else torch.bincount(idx.reshape(-1), minlength=self.n_experts).float()
        self.last_counts = counts
        if self.training and self.aux_loss_free:
            with torch.no_grad():
                if self.count_group is not None:
                    counts = counts.clone()
                    torch.distributed.all_reduce(counts, group=self.count_group)
                self.expert_bias += self.bias_update_speed * (counts.mean() - counts)
            self._aux_loss = x.new_zeros((), dtype=torch.float32)
        elif self.training:
            frac_tokens = counts / (x.shape[0] * self.topk)
            frac_probs = scores.mean(0)
            self._aux_loss = self.aux_loss_weight * self.n_experts * (frac_tokens * frac_probs).sum()
        else:
            self._aux_loss = x.new_zeros((), dtype=torch.float32)
        return w.type_as(x), idx


def share_router_counts(modules, group) -> int:
    """Make every aux-loss-free router in ``modules`` update its bias from the counts summed over ``group`` (the
    data-parallel ranks that route different tokens through the same layers): replicas then keep identical
    biases, and the step equals that of one process routing the whole global batch.  Returns the number of
    routers attached."""
    n = 0
    for m in modules:
        for sub in (m.modules() if m is not None else ()):
            if isinstance(sub, ExpertGate):
                sub.count_group = group
                n += 1
    return n


class _FusedRoute(torch.autograd.Function):
    """Router kernel forward; backward recomputes the (small) score -> weight graph in PyTorch."""

    @staticmethod
    def forward(ctx, logits, bias, k, groups, limited, sigmoid, route_scale):
        from rl_project_b200.ops._ext import native

        scores, w, idx, counts = native().moe_route(logits.contiguous(), bias, k, groups, limited, sigmoid,
                                                     route_scale)
        ctx.save_for_backward(logits, idx)
        ctx.sigmoid, ctx.route_scale = sigmoid, route_scale
        ctx.mark_non_differentiable(idx, counts)
        return w, idx, scores, counts

    @staticmethod
    def backward(ctx, dw, didx, dscores, dcounts):
        logits, idx = ctx.saved_tensors
        with torch.enable_grad():
            lg = logits.detach().requires_grad_(True)
            s = lg.sigmoid() if ctx.sigmoid else lg.softmax(-1)
            w = s.gather(1, idx)
            if ctx.sigmoid:
                w = w / (w.sum(-1, keepdim=True) + 1e-8)
            w = w * ctx.route_scale
            outs, grads = [w], [dw if dw is not None else torch.zeros_like(w)]
            if dscores is not None:
                outs.append(s)
                grads.append(dscores)
            (g,) = torch.autograd.grad(outs, [lg], grads)
        return g, None, None, None, None, None, None
