"""Rotary embeddings: frequency tables (plain/linear/YaRN) and the fused
RoPE + QKV head-split kernel (csrc/rope.cu).

Frequency rules follow ``src/forgeline/models/attention/rotary.py:11-47``
(YaRN: base rescaled by ``s^(d/(d-2))`` and a linear ramp between the
interpolated and original frequencies); ``theta`` is configurable
(``ModelSpec.rope_theta``).
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from rl_project_b200.ops._ext import native


def rope_inv_freq(dim: int, theta: float = 10000.0, scaling_type: str = "none", factor: float = 1.0,
                  max_seq_len: int = 8192) -> torch.Tensor:
    exps = torch.arange(0, dim, 2, dtype=torch.float64, device="cpu") / dim  # host, whatever the default device
    if scaling_type == "yarn" and factor != 1.0:
        base = theta * factor ** (dim / (dim - 2))
        inv = base ** (-exps)
        wavelen = 2.0 * math.pi * base ** exps
        orig_ctx = max_seq_len / factor
        ramp = ((orig_ctx / wavelen - 1.0) / (factor - 1.0)).clamp(0.0, 1.0)
        inv = inv * ((1.0 - ramp) / factor + ramp)
    else:
        inv = theta ** (-exps)
        if scaling_type == "linear":
            inv = inv / factor
    return inv.float()


class RopeTable:
    """cos/sin of ``pos * inv_freq`` as ``[max_pos, dim/2]`` fp32, grown on demand, cached per device."""

    def __init__(self, dim: int, theta: float = 10000.0, scaling_type: str = "none", factor: float = 1.0,
                 max_seq_len: int = 8192):
        self.dim = dim
        self.inv_freq = rope_inv_freq(dim, theta, scaling_type, factor, max_seq_len)
        self._rows = 0
        self._cache: dict = {}
        self._build(max(max_seq_len, 1))

    def _build(self, rows: int) -> None:
        # built on the host (a model constructed under a CUDA default device would otherwise put these on the
        # GPU at construction and on the host when the table grows later), copied to each device on use
        t = torch.arange(rows, dtype=torch.float64, device="cpu")
        ang = torch.outer(t, self.inv_freq.double().cpu())
        self._cos = ang.cos().float()
        self._sin = ang.sin().float()
        self._rows = rows
        self._cache = {}

    def tables(self, need: int, device: torch.device) -> Tuple[torch.Tensor, torch.Tensor]:
        if need > self._rows:
            self._build(max(need, 2 * self._rows))
        key = (device.type, device.index)
        if key not in self._cache:
            self._cache[key] = (self._cos.to(device), self._sin.to(device))
        return self._cache[key]


def apply_rope_reference(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: [..., T, D] with cos/sin [T, D/2] (rotate-half convention)."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    c, s = cos.to(x.device), sin.to(x.device)
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


class _RopeQKV(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cos, sin, positions, B, T, Hq, Hkv, D, offset, heads_major):
        q, k, v = native().rope_qkv_fwd(qkv, cos, sin, positions, B, T, Hq, Hkv, D, offset, heads_major)
        ctx.save_for_backward(cos, sin, positions if positions is not None else torch.empty(0))
        ctx.has_pos = positions is not None
        ctx.args = (B, T, Hq, Hkv, D, offset, heads_major)
        ctx.qkv_shape = qkv.shape
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        cos, sin, pos = ctx.saved_tensors
        B, T, Hq, Hkv, D, offset, heads_major = ctx.args
        dq = torch.zeros_like(dq) if dq is None else dq.contiguous()
        dk = torch.zeros_like(dk) if dk is None else dk.contiguous()
        dv = torch.zeros_like(dv) if dv is None else dv.contiguous()
        dqkv = native().rope_qkv_bwd(dq, dk, dv, cos, sin, pos if ctx.has_pos else None, B, T, Hq, Hkv, D, offset,
                                     heads_major)
        return dqkv.view(ctx.qkv_shape), None, None, None, None, None, None, None, None, None, None


def rope_split_qkv(qkv: torch.Tensor, table: RopeTable, n_head: int, n_kv_head: int, head_dim: int,
                   offset: int = 0, positions: Optional[torch.Tensor] = None, heads_major: bool = True,
                   rotate: bool = True, max_pos: Optional[int] = None):
    """Split ``qkv [B, T, (Hq+2Hkv)*D]`` into q/k/v (RoPE applied to q and k).

    Returns tensors of shape ``[B, H, T, D]`` (``heads_major``) or ``[B, T, H, D]``.
    ``max_pos`` (an upper bound of ``positions``, known to the caller) avoids
    reading the positions back from the device.
    """
    B, T, _ = qkv.shape
    if positions is not None:
        need = (max_pos if max_pos is not None else int(positions.max().item())) + 1
    else:
        need = offset + T
    if qkv.is_cuda and qkv.dtype == torch.bfloat16 and head_dim % 16 == 0 and rotate:
        cos, sin = table.tables(need, qkv.device)
        pos = positions.to(torch.int32).contiguous() if positions is not None else None
        return _RopeQKV.apply(qkv, cos, sin, pos, B, T, n_head, n_kv_head, head_dim, offset, heads_major)
    if qkv.is_cuda:
        native()
    q, k, v = qkv.split([n_head * head_dim, n_kv_head * head_dim, n_kv_head * head_dim], dim=-1)
    q = q.reshape(B, T, n_head, head_dim).transpose(1, 2)
    k = k.reshape(B, T, n_kv_head, head_dim).transpose(1, 2)
    v = v.reshape(B, T, n_kv_head, head_dim).transpose(1, 2)
    if rotate:
        cos, sin = table.tables(need, qkv.device)
        if positions is not None:
            c, s = cos[positions].unsqueeze(1), sin[positions].unsqueeze(1)  # [B,1,T,D/2]
        else:
            c, s = cos[offset:offset + T], sin[offset:offset + T]
        q, k = apply_rope_reference(q, c, s), apply_rope_reference(k, c, s)
    if not heads_major:
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    return q, k, v


def apply_rope(x: torch.Tensor, table: RopeTable, offset: int = 0, positions: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Rotate ``x [B, H, T, D]`` (out of place).  Used by MLA / NSA / cached decode."""
    B, H, T, D = x.shape
    need = (int(positions.max().item()) + 1) if positions is not None else offset + T
    cos, sin = table.tables(need, x.device)
    if positions is not None:
        c, s = cos[positions].unsqueeze(1), sin[positions].unsqueeze(1)
    else:
        c, s = cos[offset:offset + T], sin[offset:offset + T]
    return apply_rope_reference(x, c, s)
