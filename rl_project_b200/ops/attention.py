"""Causal self-attention entry point.

``causal_attention(q, k, v)`` with ``q [B, Hq, T, D]`` and ``k, v [B, Hkv, T, D]``
(grouped-query: ``Hq % Hkv == 0``), optional sliding window and tanh logit cap,
``q_offset`` for queries that sit after a cached prefix.  Semantics follow
``src/forgeline/models/attention/causal.py:79-134``.

``fmha_forward`` is this library's own sm_100a forward kernel (csrc/fmha_fwd.cu:
tcgen05 MMAs, TMEM accumulators, TMA loads) and ``fmha_backward`` its backward
(csrc/fmha_bwd.cu); ``fmha`` ties them together for autograd.  On CUDA (bf16,
head dim 64 or 128) windowed and soft-capped attention always runs on them; the
plain causal case runs on them when ``RLB_ATTN=tcgen05`` and otherwise on
torch's fused SDPA kernel (cuDNN / flash backends).  Dropout and the CPU path
use the explicit masked-softmax reference below.
"""

from __future__ import annotations

import math
import os
from typing import Optional, Tuple

import torch
import torch.nn.functional as F


def _expand_kv(x: torch.Tensor, rep: int) -> torch.Tensor:
    if rep == 1:
        return x
    B, H, T, D = x.shape
    return x[:, :, None].expand(B, H, rep, T, D).reshape(B, H * rep, T, D)


def attention_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int = 0, softcap: float = 0.0,
                        scale: Optional[float] = None, q_offset: Optional[int] = None,
                        causal: bool = True) -> torch.Tensor:
    B, Hq, Tq, D = q.shape
    Tk = k.shape[2]
    rep = Hq // k.shape[1]
    k, v = _expand_kv(k, rep), _expand_kv(v, rep)
    s = scale if scale is not None else 1.0 / math.sqrt(D)
    att = (q.float() @ k.float().transpose(-2, -1)) * s
    if softcap > 0:
        att = torch.tanh(att / softcap) * softcap
    off = (Tk - Tq) if q_offset is None else q_offset
    qpos = torch.arange(off, off + Tq, device=q.device)[:, None]
    kpos = torch.arange(Tk, device=q.device)[None, :]
    allowed = torch.ones(Tq, Tk, dtype=torch.bool, device=q.device)
    if causal:
        allowed &= kpos <= qpos
    if window > 0:
        allowed &= (qpos - kpos) < window
    att = att.masked_fill(~allowed, float("-inf"))
    p = torch.softmax(att, dim=-1)
    p = torch.nan_to_num(p)
    return (p @ v.float()).to(q.dtype)


_GQA_NATIVE: dict = {}


def _fused_sdpa(q, k, v, rep, dropout_p, scale):
    from torch.nn.attention import SDPBackend, sdpa_kernel

    if torch.is_grad_enabled():
        # training: fixed shapes, cuDNN's per-shape plans amortise and its kernels are the fastest here
        backends = [SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION]
    else:
        # inference prefill: shapes vary per call; the flash / memory-efficient kernels need no per-shape plan
        # (cuDNN builds one per new shape, which dominated batched prefill)
        backends = [SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION]
    key = (q.device.index, q.shape[-1], rep, torch.is_grad_enabled())
    if rep > 1 and _GQA_NATIVE.get(key, True):
        try:
            with sdpa_kernel(backends):
                out = F.scaled_dot_product_attention(q, k, v, is_causal=True, dropout_p=dropout_p, scale=scale,
                                                     enable_gqa=True)
            _GQA_NATIVE[key] = True
            return out
        except RuntimeError:
            _GQA_NATIVE[key] = False  # no fused kernel takes grouped K/V here: expand once
    with sdpa_kernel(backends):
        return F.scaled_dot_product_attention(q, _expand_kv(k, rep), _expand_kv(v, rep), is_causal=True,
                                              dropout_p=dropout_p, scale=scale)


_ATTN = os.environ.get("RLB_ATTN", "sdpa")
FMHA_SHAPES = ((64, 64), (128, 128), (192, 128))  # (d_qk, d_v) of the forward kernel; the backward: d_qk == d_v


def _token_major(x: torch.Tensor) -> torch.Tensor:
    """``[B, H, T, D]`` view -> the ``[B, T, H, D]`` tensor behind it (a copy only if it is not token-major)."""
    t = x.transpose(1, 2)
    return t if t.is_contiguous() else t.contiguous()


def fmha_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                 scale: Optional[float] = None, with_lse: bool = False, window: int = 0,
                 softcap: float = 0.0) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Attention forward on the sm_100a kernel.  ``q [B, Hq, T, D]``, ``k [B, Hkv, T, D]``, ``v [B, Hkv, T, DV]``
    (bf16; (D, DV) = (64, 64), (128, 128) or MLA's (192, 128); token-major storage avoids a copy) ->
    ``(out [B, Hq, T, DV]`` as a view of ``[B, T, Hq, DV]`` storage, ``lse [B, Hq, T]`` fp32 natural-log
    softmax denominators or None).  ``window > 0`` keeps keys with ``t - s < window``; ``softcap > 0``
    replaces each logit ``x`` by ``softcap * tanh(x / softcap)`` (the semantics of ``attention_reference``)."""
    from rl_project_b200.core.errors import KernelError
    from rl_project_b200.ops._ext import native

    B, Hq, T, D = q.shape
    DV = v.shape[-1]
    if (D, DV) not in FMHA_SHAPES or q.dtype != torch.bfloat16 or Hq % k.shape[1]:
        raise KernelError(f"fmha_forward: unsupported shape / dtype (D={D}, DV={DV}, {q.dtype}, Hq={Hq}, "
                          f"Hkv={k.shape[1]})")
    qt, kt, vt = _token_major(q), _token_major(k), _token_major(v)
    out = torch.empty(B, T, Hq, DV, dtype=q.dtype, device=q.device)
    lse = torch.empty(B, Hq, T, dtype=torch.float32, device=q.device) if with_lse else torch.empty(0, device=q.device)
    native().fmha_fwd(qt, kt, vt, out, lse, bool(causal), float(scale if scale is not None else D ** -0.5),
                      int(window), float(softcap), _status(q.device))
    return out.transpose(1, 2), (lse if with_lse else None)


def fmha_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, dout: torch.Tensor,
                  lse: torch.Tensor, causal: bool = True, scale: Optional[float] = None, window: int = 0,
                  softcap: float = 0.0):
    """Gradients of ``fmha_forward`` on the sm_100a kernel (csrc/fmha_bwd.cu): ``(dq, dk, dv)`` shaped like
    ``q, k, v`` (``[B, H, T, D]`` views of token-major storage)."""
    from rl_project_b200.ops._ext import native

    D = q.shape[-1]
    qt, kt, vt, dot = _token_major(q), _token_major(k), _token_major(v), _token_major(dout.to(torch.bfloat16))
    # Delta_t = sum_d dO * O  (the softmax-gradient row term), fp32 [B, Hq, T]
    delta = (dout.float() * out.float()).sum(-1).contiguous()
    dq = torch.empty(qt.shape, dtype=torch.float32, device=q.device)
    dk, dv = torch.empty_like(kt), torch.empty_like(vt)
    native().fmha_bwd(qt, kt, vt, dot, lse.contiguous(), delta, dq, dk, dv, bool(causal),
                      float(scale if scale is not None else D ** -0.5), int(window), float(softcap), _status(q.device))
    return dq.to(torch.bfloat16).transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2)


class _FMHA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale, window, softcap):
        out, lse = fmha_forward(q, k, v, causal, scale, with_lse=True, window=window, softcap=softcap)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.scale, ctx.window, ctx.softcap = causal, scale, window, softcap
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        dq, dk, dv = fmha_backward(q, k, v, out, dout, lse, ctx.causal, ctx.scale, ctx.window, ctx.softcap)
        return dq, dk, dv, None, None, None, None


def fmha(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
         scale: Optional[float] = None, window: int = 0, softcap: float = 0.0) -> torch.Tensor:
    """Differentiable attention on the sm_100a forward and backward kernels."""
    return _FMHA.apply(q, k, v, causal, scale, int(window), float(softcap))


_STATUS: dict = {}


def _status(device: torch.device) -> torch.Tensor:
    """Per-device status word the attention kernels report a timed-out wait into (first error kept)."""
    key = device.index
    if key not in _STATUS:
        _STATUS[key] = torch.zeros(1, dtype=torch.int32, device=device)
    return _STATUS[key]


def fmha_check(device: torch.device) -> None:
    """Raise ``KernelError`` if an attention kernel on ``device`` gave up a wait (synchronises)."""
    from rl_project_b200.core.errors import KernelError

    code = int(_status(device).item())
    if code:
        raise KernelError(f"fmha kernel: a bounded wait ran out (status 0x{code:x})",
                          hint="The GPU stalled or a kernel bug left a barrier unarrived; the output is invalid.")


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int = 0, softcap: float = 0.0,
                     scale: Optional[float] = None, dropout_p: float = 0.0) -> torch.Tensor:
    """Full-sequence causal attention (no cache).  ``q [B, Hq, T, D]`` (any strides) -> ``[B, Hq, T, D]``."""
    rep = q.shape[1] // k.shape[1]
    own = (q.is_cuda and dropout_p == 0.0 and q.dtype == torch.bfloat16 and q.shape[-1] in (64, 128)
           and v.shape[-1] == q.shape[-1])
    if own and (_ATTN == "tcgen05" or window > 0 or softcap > 0):
        # windowed / capped attention always runs on the own kernels (the masks are per-element predicates
        # there, fully masked tiles are skipped); the plain case when RLB_ATTN selects them
        if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
            return fmha(q, k, v, True, scale, window, softcap)
        return fmha_forward(q, k, v, True, scale, window=window, softcap=softcap)[0]
    if q.is_cuda and window == 0 and softcap == 0:
        return _fused_sdpa(q, k, v, rep, dropout_p, scale)
    if not q.is_cuda and window == 0 and softcap == 0 and dropout_p == 0.0:
        return F.scaled_dot_product_attention(q, _expand_kv(k, rep), _expand_kv(v, rep), is_causal=True, scale=scale)
    out = attention_reference(q, k, v, window=window, softcap=softcap, scale=scale, q_offset=0)
    if dropout_p > 0:
        out = F.dropout(out, dropout_p)
    return out
