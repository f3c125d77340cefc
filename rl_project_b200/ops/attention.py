"""Causal self-attention entry point.

``causal_attention(q, k, v)`` with ``q [B, Hq, T, D]`` and ``k, v [B, Hkv, T, D]``
(grouped-query: ``Hq % Hkv == 0``), optional sliding window and tanh logit cap,
``q_offset`` for queries that sit after a cached prefix.  Semantics follow
``src/forgeline/models/attention/causal.py:79-134``.

On CUDA, the un-windowed, un-capped case runs torch's fused SDPA kernel
(flash backend) while the sm_100a FMHA kernel is being brought up; every
other case and the CPU path use the explicit masked-softmax reference below.
"""

from __future__ import annotations

import math
from typing import Optional

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


def causal_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int = 0, softcap: float = 0.0,
                     scale: Optional[float] = None, dropout_p: float = 0.0) -> torch.Tensor:
    """Full-sequence causal attention (no cache).  ``q [B, Hq, T, D]`` (any strides) -> ``[B, Hq, T, D]``."""
    rep = q.shape[1] // k.shape[1]
    if q.is_cuda and window == 0 and softcap == 0:
        return _fused_sdpa(q, k, v, rep, dropout_p, scale)
    if not q.is_cuda and window == 0 and softcap == 0 and dropout_p == 0.0:
        return F.scaled_dot_product_attention(q, _expand_kv(k, rep), _expand_kv(v, rep), is_causal=True, scale=scale)
    out = attention_reference(q, k, v, window=window, softcap=softcap, scale=scale, q_offset=0)
    if dropout_p > 0:
        out = F.dropout(out, dropout_p)
    return out
