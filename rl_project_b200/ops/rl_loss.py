"""Clipped-surrogate + KL policy loss of GRPO / PPO in one kernel (csrc/rl_loss.cu).

``clipped_kl_loss`` returns ``(loss, policy_loss, kl)`` for per-token log-probs
``new`` (differentiable), ``old``, ``ref`` and ``mask`` of shape ``[G, R]`` and
per-sequence advantages ``adv [G]``:

* ``ratio_level`` ``sequence_mean``: ``r = exp(masked_mean(new - old))`` per
  sequence; ``token``: ``r_t = exp(new_t - old_t)`` and the surrogate is
  masked-averaged per sequence;
* ``kl``: ``logprob_diff`` -- ``clamp(mean_g(masked_mean(ref - new)), 0)``
  (GRPO, ``src/forgeline/training/grpo.py:177-180``); ``logprob_diff_rows`` --
  ``mean_g(clamp(masked_mean(ref - new), 0))`` (PPO); ``k3`` --
  ``mean_g(masked_mean(exp(d) - d - 1))``, ``d = ref - new``.

On CUDA the kernel forms the per-sequence terms and the gradient with respect
to ``new`` in one pass; backward is a single scale.  Elsewhere the same
formulas run as PyTorch ops (the reference's own composition).
"""

from __future__ import annotations

import torch

from rl_project_b200.ops._ext import available, native

KL_MODES = ("logprob_diff", "logprob_diff_rows", "k3")


def _masked_mean(x, m):
    return (x * m).sum(-1) / m.sum(-1).clamp(min=1.0)


def clipped_kl_loss_reference(new, old, ref, mask, adv, clip: float, kl_coef: float, ratio_level: str,
                              kl: str):
    m = mask.to(new.dtype)
    if ratio_level == "sequence_mean":
        r = torch.exp(_masked_mean(new - old, m))
        pl = -torch.min(r * adv, torch.clamp(r, 1 - clip, 1 + clip) * adv)
    else:
        r = torch.exp(new - old)
        a = adv[:, None]
        pl = _masked_mean(-torch.min(r * a, torch.clamp(r, 1 - clip, 1 + clip) * a), m)
    pl = pl.mean()
    d = ref - new
    if kl == "k3":
        klv = _masked_mean(torch.exp(d) - d - 1.0, m).mean()
    elif kl == "logprob_diff_rows":
        klv = _masked_mean(d, m).clamp(min=0).mean()
    else:
        klv = _masked_mean(d, m).mean().clamp(min=0)
    return pl + kl_coef * klv, pl, klv


class _ClippedKL(torch.autograd.Function):
    @staticmethod
    def forward(ctx, new, old, ref, mask, adv, clip, kl_coef, token_level, kl):
        pl_row, kl_row, dpl, dkl = native().rl_loss(new.contiguous(), old.contiguous(), ref.contiguous(),
                                                    mask.contiguous(), adv.contiguous(), clip, token_level,
                                                    kl == "k3")
        G = new.shape[0]
        pl = pl_row.mean()
        if kl == "k3":
            klv = kl_row.mean()
            act = torch.ones(G, 1, device=new.device)
        elif kl == "logprob_diff_rows":
            klv = kl_row.clamp(min=0).mean()
            act = (kl_row >= 0).float()[:, None]
        else:
            mean = kl_row.mean()
            klv = mean.clamp(min=0)
            act = (mean >= 0).float().expand(G)[:, None]
        ctx.save_for_backward(dpl, dkl, act)
        ctx.kl_coef, ctx.G = kl_coef, G
        ctx.mark_non_differentiable(pl, klv)
        return pl + kl_coef * klv, pl, klv

    @staticmethod
    def backward(ctx, g_loss, g_pl, g_kl):
        dpl, dkl, act = ctx.saved_tensors
        dnew = (dpl + (ctx.kl_coef * act) * dkl) * (g_loss / ctx.G)
        return dnew, None, None, None, None, None, None, None, None


def clipped_kl_loss(new, old, ref, mask, adv, clip: float, kl_coef: float, ratio_level: str = "sequence_mean",
                    kl: str = "logprob_diff"):
    """-> ``(loss, policy_loss, kl)``; see the module docstring for the terms."""
    if kl not in KL_MODES:
        raise ValueError(f"kl must be one of {KL_MODES}, got {kl!r}")
    if ratio_level not in ("sequence_mean", "token"):
        raise ValueError(f"ratio_level must be sequence_mean|token, got {ratio_level!r}")
    if new.is_cuda and available() and new.dim() == 2:
        f = torch.float32
        return _ClippedKL.apply(new.to(f), old.to(f), ref.to(f), mask.to(f), adv.to(f), float(clip), float(kl_coef),
                                ratio_level == "token", kl)
    return clipped_kl_loss_reference(new, old, ref, mask, adv, clip, kl_coef, ratio_level, kl)
