"""Mixture-of-experts layer with sort-based dispatch.

The reference loops ``topk x n_experts`` with boolean masks
(``src/forgeline/models/moe/layer.py:32-38``).  Here the (token, slot) pairs
are sorted by expert once and the weighted outputs are scattered back with
one ``index_add_``.  On CUDA the experts run as grouped tcgen05 GEMMs over a
padded expert-sorted buffer (rl_project_b200/ops/grouped_gemm.py): three
launches per layer and pass whatever the expert count, with no host
synchronisation; elsewhere each expert runs on its contiguous segment.  The same
permutation feeds the expert-parallel all-to-all (parallel/expert.py).
Parameter names (``gate``, ``experts.{e}.w*``, ``shared_experts.w*``) match
the reference checkpoints.
"""

from __future__ import annotations

import os
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

    # ------------------------------------------------------------------ grouped-GEMM path (CUDA)
    def _grouped_ready(self, xs: torch.Tensor) -> bool:
        from rl_project_b200.models.transformer.feedforward import SwiGLUFeedForward
        from rl_project_b200.ops._ext import available

        if not (xs.is_cuda and xs.dtype == torch.bfloat16 and available()):
            return False
        if os.environ.get("RLB_MOE_GROUPED", "1") == "0":  # per-expert loop, for A/B measurements
            return False
        m = next((e for e in self.experts if isinstance(e, SwiGLUFeedForward)), None)
        if m is None or not m._fusable() or type(m.w2) is not nn.Linear or m.w2.bias is not None:
            return False
        F, C = m.hidden_dim, xs.shape[1]
        return C % 64 == 0 and F % 32 == 0 and m.w1.weight.dtype == torch.bfloat16

    def _stacked(self, first: int, n: int):
        """Stacked ``w13 [n, 2F, C]`` and ``w2 [n, C, F]`` of experts ``first..first+n`` and the parameters whose
        gradients they carry.  The first call moves the experts' weights into two packed buffers (each
        parameter becomes a view), so later calls cost nothing; parameters that live in someone else's
        flat buffer (sharded data parallel) are stacked by copying instead, with gradients through autograd."""
        mods = [self.experts[first + j] for j in range(n)]
        params = [m.w1.weight for m in mods] + [m.w3.weight for m in mods] + [m.w2.weight for m in mods]
        pk = getattr(self, "_pack", None)
        if pk is not None and pk["key"] == (first, n) and all(
                p.data_ptr() == q for p, q in zip(params, pk["ptrs"])):
            return pk["w13"], pk["w2"], params
        own = all(p.untyped_storage().nbytes() == p.numel() * p.element_size() for p in params)
        if not own:
            w13 = torch.stack([torch.cat([m.w1.weight, m.w3.weight], 0) for m in mods])
            w2 = torch.stack([m.w2.weight for m in mods])
            return w13, w2, ()
        F, C = mods[0].hidden_dim, mods[0].w1.weight.shape[1]
        dev, dt = params[0].device, params[0].dtype
        w13 = torch.empty(n, 2 * F, C, device=dev, dtype=dt)
        w2 = torch.empty(n, C, F, device=dev, dtype=dt)
        with torch.no_grad():
            for j, m in enumerate(mods):
                w13[j, :F].copy_(m.w1.weight)
                w13[j, F:].copy_(m.w3.weight)
                w2[j].copy_(m.w2.weight)
                m.w1.weight.data = w13[j, :F]
                m.w3.weight.data = w13[j, F:]
                m.w2.weight.data = w2[j]
        self._pack = {"key": (first, n), "w13": w13, "w2": w2, "ptrs": [p.data_ptr() for p in params]}
        return w13, w2, params

    def _experts_grouped(self, xp: torch.Tensor, layout, first: int, n: int) -> torch.Tensor:
        from rl_project_b200.ops.grouped_gemm import grouped_swiglu_experts

        w13, w2, params = self._stacked(first, n)
        sink = self._pack if params else None
        return grouped_swiglu_experts(xp, layout, w13, w2, params, sink)

    def _run_grouped(self, xs: torch.Tensor, counts: torch.Tensor, sorted_experts: torch.Tensor,
                     first: int) -> torch.Tensor:
        """Rows already sorted by expert (expert-parallel receive buffer) through the grouped experts."""
        from rl_project_b200.ops.grouped_gemm import grouped_layout
        from rl_project_b200.ops.moe_dispatch import combine, dispatch, row_maps

        layout = grouped_layout(sorted_experts, counts)
        order = torch.arange(xs.shape[0], device=xs.device)
        maps = row_maps(order, layout.dest, layout.rows, 1)
        y = self._experts_grouped(dispatch(xs, maps), layout, first, counts.numel())
        return combine(y, torch.ones(xs.shape[0], 1, device=xs.device, dtype=torch.float32), maps)

    def _forward_grouped(self, xf: torch.Tensor, weights: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        """Route, dispatch into the padded expert-sorted buffer, run the grouped experts and combine: every
        step is a device op (no host synchronisation) and both directions are gathers (no atomics)."""
        from rl_project_b200.ops.grouped_gemm import grouped_layout
        from rl_project_b200.ops.moe_dispatch import combine, dispatch, row_maps

        k = indices.shape[1]
        flat = indices.reshape(-1)
        order = torch.sort(flat, stable=True).indices
        counts = torch.bincount(flat, minlength=self.n_experts)
        layout = grouped_layout(flat.index_select(0, order), counts)
        maps = row_maps(order, layout.dest, layout.rows, k)
        y = self._experts_grouped(dispatch(xf, maps), layout, 0, self.n_experts)
        return combine(y, weights, maps)

    def run_experts(self, xs: torch.Tensor, counts: List[int], first_expert: int = 0) -> torch.Tensor:
        if self._grouped_ready(xs):
            ct = torch.as_tensor(counts, device=xs.device, dtype=torch.int64)
            se = torch.repeat_interleave(torch.arange(len(counts), device=xs.device), ct, output_size=xs.shape[0])
            return self._run_grouped(xs, ct, se, first_expert)
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
        elif self._grouped_ready(xf):
            y = self._forward_grouped(xf, weights, indices)
        else:
            order, tok, counts = sort_by_expert(indices, self.n_experts)
            xs = xf.index_select(0, tok)
            ys = self.run_experts(xs, counts.tolist())
            w = weights.reshape(-1).index_select(0, order).unsqueeze(-1).to(ys.dtype)
            y = torch.zeros_like(xf).index_add_(0, tok, ys * w)
        if self.shared_experts is not None:
            y = y + self.shared_experts(xf)
        return y.view(B, T, C)
