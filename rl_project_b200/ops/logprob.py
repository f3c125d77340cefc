"""Fused LM-head -> log-softmax -> gather (kernel: csrc/logprob.cu).

``linear_logprobs(h, W, targets)`` returns per-token ``log p(target)`` (and
optionally the entropy) without ever building an fp32 ``[N, V]`` tensor:
logits exist only in bf16; when the own GEMM runs the LM-head forward its
epilogue also writes each row's online log-sum-exp statistics per 256-column
chunk, so a small merge pass gives the outputs without re-reading the logits
(otherwise the kernel makes ONE pass over each row for the forward), and the
backward rewrites the same buffer in
place with ``g * (onehot - softmax)`` before the two GEMMs that produce
``dh`` and ``dW``.  When ``N * V`` bf16 logits exceed the keep budget, rows
are processed in chunks and recomputed in backward.

Replaces ``F.cross_entropy`` at ``src/forgeline/models/transformer/model.py:154``
and ``token_logprobs_from_logits`` at ``src/forgeline/models/policy.py:47-50``.
"""

from __future__ import annotations

import os
from typing import List, Optional, Tuple

import torch
import torch.nn.functional as F

from rl_project_b200.ops._ext import native

KEEP_BUDGET_BYTES = int(float(os.environ.get("RLB_LOGITS_KEEP_GB", "24")) * (1 << 30))
CHUNK_ROWS = int(os.environ.get("RLB_LOGITS_CHUNK_ROWS", "16384"))


from rl_project_b200.ops.linear import matmul_nn, matmul_tn  # noqa: E402


def _gemm_nt(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a [M, K] @ b[N, K]^T -> [M, N]."""
    from rl_project_b200.ops.linear import matmul_nt

    return matmul_nt(a, b)


class _LinearLogprob(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, W, targets, with_entropy):
        N = h.shape[0]
        V = W.shape[0]
        keep = N * V * 2 <= KEEP_BUDGET_BYTES
        step = N if keep else max(1, min(N, CHUNK_ROWS))
        lse_parts, lp_parts, ent_parts, kept = [], [], [], []
        from rl_project_b200.ops import gemm

        for s in range(0, N, step):
            hs = h[s:s + step]
            if hs.is_cuda and gemm.lse_fusable(hs, W):
                # the GEMM's epilogue writes per-chunk row statistics: no second pass over the logits
                logits, stats = gemm.gemm_nt_lse(hs, W)
                outs = native().logprob_combine(stats, logits, targets[s:s + step], with_entropy, None)
            else:
                logits = _gemm_nt(hs, W)
                outs = native().logprob_fwd(logits, targets[s:s + step], with_entropy, None)
            lse_parts.append(outs[0])
            lp_parts.append(outs[1])
            if with_entropy:
                ent_parts.append(outs[2])
            if keep:
                kept.append(logits)
        lse = torch.cat(lse_parts)
        lp = torch.cat(lp_parts)
        ent = torch.cat(ent_parts) if with_entropy else None
        ctx.keep = keep
        ctx.step = step
        ctx.with_entropy = with_entropy
        ctx.kept = kept
        ctx.save_for_backward(h, W, targets, lse, ent if ent is not None else torch.empty(0))
        ctx.mark_non_differentiable(lse)
        if with_entropy:
            return lp, ent
        return lp, lse

    @staticmethod
    def backward(ctx, g_lp, g_second):
        h, W, targets, lse, ent = ctx.saved_tensors
        g_ent = g_second if ctx.with_entropy else None
        N = h.shape[0]
        step = ctx.step
        dh = torch.empty_like(h)
        dW32: Optional[torch.Tensor] = None
        dW16: Optional[torch.Tensor] = None
        g_lp = g_lp.float().contiguous() if g_lp is not None else None
        g_ent = g_ent.float().contiguous() if g_ent is not None else None
        for i, s in enumerate(range(0, N, step)):
            logits = ctx.kept[i] if ctx.keep else _gemm_nt(h[s:s + step], W)
            native().logprob_bwd_(logits, targets[s:s + step], lse[s:s + step],
                                  g_lp[s:s + step] if g_lp is not None else None,
                                  ent[s:s + step] if ctx.with_entropy else None,
                                  g_ent[s:s + step] if g_ent is not None else None, 1.0)
            dh[s:s + step] = matmul_nn(logits, W)
            part = matmul_tn(logits, h[s:s + step])
            if N <= step:
                dW16 = part
            else:
                dW32 = part.float() if dW32 is None else dW32.add_(part.float())
            del logits
        ctx.kept = []
        dW = dW16 if dW16 is not None else dW32.to(W.dtype)
        return dh, dW, None, None


def linear_logprobs_reference(h: torch.Tensor, W: torch.Tensor, targets: torch.Tensor, with_entropy: bool = False):
    logits = (h.float() @ W.float().t())
    logp = torch.log_softmax(logits, dim=-1)
    safe = targets.clamp(min=0)
    lp = logp.gather(-1, safe.unsqueeze(-1)).squeeze(-1) * (targets >= 0).float()
    if with_entropy:
        ent = -(logp.exp() * logp).sum(-1)
        return lp, ent
    return lp, torch.logsumexp(logits, dim=-1)


def linear_logprobs(h: torch.Tensor, W: torch.Tensor, targets: torch.Tensor,
                    with_entropy: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """``h [N, d]``, ``W [V, d]``, ``targets [N]`` (-1 = ignore) -> ``(lp [N], lse [N] | entropy [N])``."""
    targets = targets.reshape(-1).to(torch.long).contiguous()
    h2 = h.reshape(-1, h.shape[-1])
    if h2.is_cuda and h2.dtype == torch.bfloat16:
        Wc = W if W.dtype == torch.bfloat16 else W.to(torch.bfloat16)
        return _LinearLogprob.apply(h2.contiguous(), Wc, targets, with_entropy)
    if h2.is_cuda:
        native()
    return linear_logprobs_reference(h2, W, targets, with_entropy)


def linear_cross_entropy(h: torch.Tensor, W: torch.Tensor, targets: torch.Tensor,
                         ignore_index: int = -1) -> torch.Tensor:
    """Mean token cross-entropy of ``h @ W^T`` against ``targets`` (``ignore_index`` skipped)."""
    t = targets.reshape(-1).to(torch.long)
    if ignore_index != -1:
        t = torch.where(t == ignore_index, torch.full_like(t, -1), t)
    lp, _ = linear_logprobs(h, W, t)
    n = (t >= 0).sum().clamp(min=1)
    return -(lp.sum() / n)


def logprobs_from_logits(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Token log-probs from already materialised logits ``[..., V]`` (any device)."""
    flat = logits.reshape(-1, logits.shape[-1])
    t = targets.reshape(-1).to(torch.long)
    lp = -F.cross_entropy(flat.float(), t, reduction="none", ignore_index=-1)
    return lp.view(targets.shape)
