"""RMSNorm and fused residual-add + RMSNorm (kernel: csrc/norm.cu).

Reference semantics: ``src/forgeline/models/transformer/norm.py:9-17``.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from rl_project_b200.ops._ext import native


def rms_norm_reference(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        y, rstd = native().rmsnorm_fwd(x2, None, w, eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dx, dw = native().rmsnorm_bwd(x2, w, rstd, dy.reshape(x2.shape).contiguous(), None)
        return dx.view(ctx.shape), dw, None


class _AddRMSNorm(torch.autograd.Function):
    """h = x + delta; y = rmsnorm(h).  Returns (h, y)."""

    @staticmethod
    def forward(ctx, x, delta, w, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        d2 = delta.reshape(-1, shape[-1]).contiguous()
        y, rstd, h = native().rmsnorm_fwd(x2, d2, w, eps)
        ctx.save_for_backward(h, w, rstd)
        ctx.shape = shape
        return h.view(shape), y.view(shape)

    @staticmethod
    def backward(ctx, dh, dy):
        h, w, rstd = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(h)
        dres = None if dh is None else dh.reshape(h.shape).contiguous()
        dx, dw = native().rmsnorm_bwd(h, w, rstd, dy.reshape(h.shape).contiguous(), dres)
        dx = dx.view(ctx.shape)
        return dx, dx, dw, None


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    if x.is_cuda and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0:
        return _RMSNorm.apply(x, w.to(torch.bfloat16) if w.dtype != torch.bfloat16 else w, eps)
    if x.is_cuda:
        native()  # fail loudly when the library is missing on a GPU
    return rms_norm_reference(x, w, eps)


def add_rms_norm(x: torch.Tensor, delta: torch.Tensor, w: torch.Tensor, eps: float = 1e-6) -> Tuple[torch.Tensor, torch.Tensor]:
    if x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0:
        return _AddRMSNorm.apply(x, delta, w, eps)
    h = x + delta
    return h, rms_norm(h, w, eps)
