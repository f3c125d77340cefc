"""Feed-forward blocks (``src/forgeline/models/transformer/feedforward.py:14-44``).

``SwiGLUFeedForward`` keeps the reference's ``w1``/``w2``/``w3`` parameters
(checkpoint keys) but runs ``w1`` and ``w3`` as ONE GEMM over the
concatenated weight, followed by the fused SwiGLU kernel -- or, with the own GEMM enabled, as one GEMM
whose epilogue applies the activation.  The hidden width
is ``hidden_dim`` (``ModelSpec.d_ff``) or the reference's derived width.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.ops import gemm
from rl_project_b200.ops.activation import gelu_tanh, swiglu
from rl_project_b200.ops.linear import linear


def default_swiglu_hidden(dim: int) -> int:
    raw = int(8 * dim / 3)
    return 64 * ((raw + 63) // 64)


class SwiGLUFeedForward(nn.Module):
    def __init__(self, dim: int, hidden_dim: Optional[int] = None, bias: bool = False, dropout: float = 0.0):
        super().__init__()
        hidden_dim = hidden_dim or default_swiglu_hidden(dim)
        self.hidden_dim = hidden_dim
        self.w1 = nn.Linear(dim, hidden_dim, bias=bias)
        self.w2 = nn.Linear(hidden_dim, dim, bias=bias)
        self.w3 = nn.Linear(dim, hidden_dim, bias=bias)
        self.dropout = nn.Dropout(dropout)
        self.tp_group = None  # set by tensor parallelism (hidden width then split over the group)

    def _fusable(self) -> bool:
        return type(self.w1) is nn.Linear and type(self.w3) is nn.Linear and self.w1.bias is None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp_group is not None:
            from rl_project_b200.parallel.tensor_parallel import column_parallel_in, copy_to_tp, row_parallel_out
        if self._fusable():
            w13 = torch.cat([self.w1.weight, self.w3.weight], dim=0)
            if self.tp_group is None and x.is_cuda and gemm.swiglu_fusable(x.reshape(-1, x.shape[-1]), w13):
                if type(self.w2) is nn.Linear and self.w2.bias is None:
                    # forward activation and its backward both in GEMM epilogues
                    return self.dropout(gemm.swiglu_ffn(x, w13, self.w2.weight))
                a = gemm.linear_swiglu(x, w13)  # activation in the GEMM epilogue
            else:
                h13 = column_parallel_in(x, w13, None, self.tp_group) if self.tp_group is not None else linear(x, w13)
                a = swiglu(h13)
        else:  # adapters wrap w1/w3: run them as modules
            if self.tp_group is not None:
                x = copy_to_tp(x, self.tp_group)
            a = swiglu(torch.cat([self.w1(x), self.w3(x)], dim=-1))
        if self.tp_group is not None:
            out = row_parallel_out(a, self.w2, self.tp_group)
        else:
            out = self.w2(a) if type(self.w2) is not nn.Linear else linear(a, self.w2.weight, self.w2.bias)
        return self.dropout(out)


class GELUFeedForward(nn.Module):
    def __init__(self, dim: int, hidden_dim: Optional[int] = None, bias: bool = False, dropout: float = 0.0):
        super().__init__()
        hidden_dim = hidden_dim or 4 * dim
        self.c_fc = nn.Linear(dim, hidden_dim, bias=bias)
        self.c_proj = nn.Linear(hidden_dim, dim, bias=bias)
        self.dropout = nn.Dropout(dropout)
        self.tp_group = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp_group is None:
            return self.dropout(self.c_proj(gelu_tanh(self.c_fc(x))))
        from rl_project_b200.parallel.tensor_parallel import column_parallel_in, copy_to_tp, row_parallel_out

        if type(self.c_fc) is nn.Linear:
            h = gelu_tanh(column_parallel_in(x, self.c_fc.weight, self.c_fc.bias, self.tp_group))
        else:
            h = gelu_tanh(self.c_fc(copy_to_tp(x, self.tp_group)))
        return self.dropout(row_parallel_out(h, self.c_proj, self.tp_group))


def make_ffn(spec: ModelSpec, hidden_dim: Optional[int] = None) -> nn.Module:
    if spec.use_swiglu:
        return SwiGLUFeedForward(spec.n_embd, hidden_dim or spec.ffn_hidden, spec.bias, spec.dropout)
    return GELUFeedForward(spec.n_embd, hidden_dim or spec.ffn_hidden, spec.bias, spec.dropout)
