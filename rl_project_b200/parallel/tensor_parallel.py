"""Megatron-style 1-D tensor parallelism with head-divided attention.

``apply_tensor_parallel`` shards a ``TransformerLM`` in place over a TP group:

* attention: q / k / v projections are split by heads (each rank keeps
  ``n_head / tp`` query heads and ``n_kv_head / tp`` KV heads and runs
  attention on them alone -- the head counts of the module are divided, unlike
  the reference's ``src/forgeline/distributed/tensor_parallel.py:14-129``,
  which kept global head counts); the output projection is split by input
  columns;
* SwiGLU / GELU feed-forward: ``w1``/``w3`` (``c_fc``) split by output rows,
  ``w2`` (``c_proj``) by input columns.

Each sharded module gets ``tp_group``: its forward applies ``copy_to_tp``
(identity forward, all-reduce of the input gradient backward) on entry and
``reduce_from_tp`` (all-reduce forward, identity backward) after the row-split
projection, adding a bias once after the reduction.  On NCCL GPU ranks the
row-split projection and its all-reduce are one tcgen05 GEMM that reduces
over peer memory in its epilogue (parallel/tp_fused.py).  Norms, embeddings and the
LM head stay replicated: their inputs and gradients are identical on every TP
rank, so they need no synchronisation.  Every rank of a TP group must see the
same micro-batch.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

from rl_project_b200.core.errors import DistributedConfigError


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous().clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        x = x.contiguous().clone()
        dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


def copy_to_tp(x: torch.Tensor, group: Any) -> torch.Tensor:
    return _CopyToTP.apply(x, group)


def reduce_from_tp(x: torch.Tensor, group: Any) -> torch.Tensor:
    return _ReduceFromTP.apply(x, group)


def _slice_linear(lin: nn.Linear, dim: int, lo: int, hi: int, keep_bias: bool) -> nn.Linear:
    """A new ``nn.Linear`` holding rows (dim 0) or columns (dim 1) ``[lo, hi)`` of ``lin``."""
    w = lin.weight.detach()
    w = w[lo:hi] if dim == 0 else w[:, lo:hi]
    out = nn.Linear(w.shape[1], w.shape[0], bias=lin.bias is not None, device=w.device, dtype=w.dtype)
    with torch.no_grad():
        out.weight.copy_(w)
        if lin.bias is not None:
            if dim == 0:
                out.bias.copy_(lin.bias.detach()[lo:hi])
            elif keep_bias:
                out.bias.copy_(lin.bias.detach())
    return out


def _rows(lin: nn.Linear, rank: int, size: int) -> nn.Linear:
    n = lin.out_features // size
    return _slice_linear(lin, 0, rank * n, (rank + 1) * n, True)


def _cols(lin: nn.Linear, rank: int, size: int) -> nn.Linear:
    n = lin.in_features // size
    return _slice_linear(lin, 1, rank * n, (rank + 1) * n, True)


def shard_attention(attn: nn.Module, group: Any, rank: int, size: int) -> None:
    from rl_project_b200.models.attention.causal import CausalSelfAttention

    if type(attn) is not CausalSelfAttention:
        raise DistributedConfigError(f"tensor parallelism supports grouped-query attention, not {type(attn).__name__}",
                                     hint="Use expert/data parallelism for MLA / NSA models.")
    H, Hkv, D = attn.n_head, attn.n_kv_head, attn.head_dim
    if H % size or Hkv % size:
        raise DistributedConfigError(f"n_head {H} and n_kv_head {Hkv} must be divisible by tensor_parallel {size}")
    hq, hk = H // size, Hkv // size
    attn.q_proj = _slice_linear(attn.q_proj, 0, rank * hq * D, (rank + 1) * hq * D, True)
    attn.k_proj = _slice_linear(attn.k_proj, 0, rank * hk * D, (rank + 1) * hk * D, True)
    attn.v_proj = _slice_linear(attn.v_proj, 0, rank * hk * D, (rank + 1) * hk * D, True)
    attn.c_proj = _cols(attn.c_proj, rank, size)
    attn.n_head, attn.n_kv_head = hq, hk
    attn.tp_group = group


def shard_ffn(ffn: nn.Module, group: Any, rank: int, size: int) -> None:
    from rl_project_b200.models.transformer.feedforward import GELUFeedForward, SwiGLUFeedForward

    if type(ffn) is SwiGLUFeedForward:
        if ffn.hidden_dim % size:
            raise DistributedConfigError(f"ffn hidden {ffn.hidden_dim} not divisible by tensor_parallel {size}")
        ffn.w1, ffn.w3, ffn.w2 = _rows(ffn.w1, rank, size), _rows(ffn.w3, rank, size), _cols(ffn.w2, rank, size)
        ffn.hidden_dim //= size
    elif type(ffn) is GELUFeedForward:
        ffn.c_fc, ffn.c_proj = _rows(ffn.c_fc, rank, size), _cols(ffn.c_proj, rank, size)
    else:
        raise DistributedConfigError(f"tensor parallelism does not shard {type(ffn).__name__}",
                                     hint="MoE layers scale with expert_parallel instead.")
    ffn.tp_group = group


def apply_tensor_parallel(model: nn.Module, group: Any, rank: int, size: int) -> nn.Module:
    """Shard every block of ``model`` over the TP group (in place); returns the model."""
    if size == 1:
        return model
    for blk in model.transformer.h:
        shard_attention(blk.attn, group, rank, size)
        shard_ffn(blk.ffn, group, rank, size)
    model.tp_size = size
    return model


def row_parallel_out(x: torch.Tensor, lin: nn.Module, group: Any) -> torch.Tensor:
    """``lin(x)`` for a column-split ``lin``: local GEMM, all-reduce over the group, bias once."""
    from rl_project_b200.ops.linear import linear
    from rl_project_b200.parallel.tp_fused import reducer_for, row_parallel_linear_fused

    if type(lin) is nn.Linear:
        reducer = reducer_for(group, x.reshape(-1, x.shape[-1]), lin.weight.shape[0])
        if reducer is not None:  # GEMM with the all-reduce in its epilogue (peer memory, tile by tile)
            y = row_parallel_linear_fused(x, lin.weight, reducer)
            return y + lin.bias if lin.bias is not None else y
        y = linear(x, lin.weight, None)
    else:
        y = nn.functional.linear(x, lin.weight)
    y = reduce_from_tp(y, group)
    return y + lin.bias if getattr(lin, "bias", None) is not None else y


def column_parallel_in(x: torch.Tensor, w: torch.Tensor, bias: Any, group: Any) -> torch.Tensor:
    """``copy_to_tp(x) @ w^T (+ bias)`` for a row-split ``w``: on NCCL GPU ranks with the fused reducer,
    the backward all-reduce of ``dx`` runs inside the dgrad GEMM's epilogue."""
    from rl_project_b200.ops.linear import linear
    from rl_project_b200.parallel.tp_fused import column_parallel_linear_fused, reducer_for

    reducer = reducer_for(group, x.reshape(-1, x.shape[-1]), x.shape[-1]) if w.dtype == torch.bfloat16 else None
    if reducer is not None:
        y = column_parallel_linear_fused(x, w, reducer)
        return y + bias if bias is not None else y
    return linear(copy_to_tp(x, group), w, bias)


# ---------------------------------------------------------------- reference-compatible layer API
# (src/forgeline/distributed/tensor_parallel.py:39-129 names: all_reduce_forward / all_reduce_backward,
# ColumnParallelLinear, RowParallelLinear with ``from_linear``), built on the collectives above.

def all_reduce_forward(x: torch.Tensor, group: Any) -> torch.Tensor:
    """All-reduce in forward, identity in backward (the row-parallel output)."""
    return reduce_from_tp(x, group)


def all_reduce_backward(x: torch.Tensor, group: Any) -> torch.Tensor:
    """Identity in forward, all-reduce of the gradient in backward (the column-parallel input)."""
    return copy_to_tp(x, group)


class ColumnParallelLinear(nn.Module):
    """Linear layer whose output features are split over the TP group (rank r keeps rows
    ``[r out/tp, (r+1) out/tp)``); ``gather_output`` concatenates the shards (differentiable)."""

    def __init__(self, in_features: int, out_features: int, tp_group: Any, tp_size: int, bias: bool = False,
                 gather_output: bool = False):
        super().__init__()
        if out_features % tp_size:
            raise DistributedConfigError(f"out_features {out_features} not divisible by tensor_parallel {tp_size}")
        self.in_features, self.out_features = in_features, out_features
        self.tp_group, self.tp_size, self.gather_output = tp_group, tp_size, gather_output
        self.weight = nn.Parameter(torch.empty(out_features // tp_size, in_features))
        self.bias = nn.Parameter(torch.zeros(out_features // tp_size)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)

    @classmethod
    def from_linear(cls, linear: nn.Linear, tp_group: Any, tp_size: int, tp_rank: int) -> "ColumnParallelLinear":
        layer = cls(linear.in_features, linear.out_features, tp_group, tp_size, linear.bias is not None)
        src = _rows(linear, tp_rank, tp_size)
        with torch.no_grad():
            layer.weight.copy_(src.weight)
            if layer.bias is not None:
                layer.bias.copy_(src.bias)
        return layer.to(linear.weight.device, linear.weight.dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from rl_project_b200.ops.linear import linear

        y = linear(copy_to_tp(x, self.tp_group), self.weight, self.bias)
        if self.gather_output and self.tp_size > 1:
            import torch.distributed.nn.functional as dnnf

            y = torch.cat(dnnf.all_gather(y.contiguous(), group=self.tp_group), dim=-1)
        return y


class RowParallelLinear(nn.Module):
    """Linear layer whose input features are split over the TP group: local product, all-reduce (the fused
    GEMM epilogue on GPU ranks when enabled), bias added once."""

    def __init__(self, in_features: int, out_features: int, tp_group: Any, tp_size: int, bias: bool = False):
        super().__init__()
        if in_features % tp_size:
            raise DistributedConfigError(f"in_features {in_features} not divisible by tensor_parallel {tp_size}")
        self.in_features, self.out_features = in_features, out_features
        self.tp_group, self.tp_size = tp_group, tp_size
        self.weight = nn.Parameter(torch.empty(out_features, in_features // tp_size))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)

    @classmethod
    def from_linear(cls, linear: nn.Linear, tp_group: Any, tp_size: int, tp_rank: int) -> "RowParallelLinear":
        layer = cls(linear.in_features, linear.out_features, tp_group, tp_size, linear.bias is not None)
        src = _cols(linear, tp_rank, tp_size)
        with torch.no_grad():
            layer.weight.copy_(src.weight)
            if layer.bias is not None:
                layer.bias.copy_(src.bias)
        return layer.to(linear.weight.device, linear.weight.dtype)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return row_parallel_out(x, self, self.tp_group)
