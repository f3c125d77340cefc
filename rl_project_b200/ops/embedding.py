"""Token-embedding gather with a deterministic sorted-segment backward (csrc/embedding.cu)."""

from __future__ import annotations

import torch
import torch.nn.functional as F

from rl_project_b200.ops._ext import native


class _Embed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, idx, W):
        ctx.save_for_backward(idx)
        ctx.vocab = W.shape[0]
        return native().embed_fwd(idx, W, None)

    @staticmethod
    def backward(ctx, dy):
        (idx,) = ctx.saved_tensors
        dW = native().embed_bwd(idx, dy.reshape(-1, dy.shape[-1]).contiguous(), ctx.vocab)
        return None, dW


def embedding(idx: torch.Tensor, W: torch.Tensor) -> torch.Tensor:
    if W.is_cuda and W.dtype == torch.bfloat16 and W.shape[1] % 8 == 0:
        return _Embed.apply(idx.to(torch.long).contiguous(), W)
    if W.is_cuda:
        native()
    return F.embedding(idx, W)
