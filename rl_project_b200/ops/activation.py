"""SwiGLU / GELU activations (kernel: csrc/swiglu.cu).

Reference: ``src/forgeline/models/transformer/feedforward.py:14-44``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from rl_project_b200.ops._ext import native


def swiglu_reference(h13: torch.Tensor) -> torch.Tensor:
    g, u = h13.chunk(2, dim=-1)
    return F.silu(g) * u


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h13):
        h13 = h13.contiguous()
        ctx.save_for_backward(h13)
        return native().swiglu_fwd(h13)

    @staticmethod
    def backward(ctx, da):
        (h13,) = ctx.saved_tensors
        return native().swiglu_bwd(h13, da.contiguous())


def swiglu(h13: torch.Tensor) -> torch.Tensor:
    """``silu(h13[..., :F]) * h13[..., F:]`` for a fused [gate | up] projection."""
    if h13.is_cuda and h13.dtype == torch.bfloat16 and (h13.shape[-1] // 2) % 8 == 0:
        return _SwiGLU.apply(h13)
    if h13.is_cuda:
        native()
    return swiglu_reference(h13)


class _GELU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        x = x.contiguous()
        ctx.save_for_backward(x)
        return native().gelu(x, None)

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        return native().gelu(x, dy.contiguous())


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    if x.is_cuda and x.dtype == torch.bfloat16 and x.numel() % 8 == 0:
        return _GELU.apply(x)
    return F.gelu(x, approximate="tanh")
