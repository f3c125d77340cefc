"""Native sparse attention (``src/forgeline/models/attention/sparse.py:16-118``):
compressed-block, top-k selected and sliding-window branches mixed by a
learned per-head softmax gate.  Like the reference, no cached decode."""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.ops.rope import RopeTable, apply_rope


class NativeSparseAttention(nn.Module):
    def __init__(self, spec: ModelSpec):
        super().__init__()
        self.n_head = spec.n_head
        self.head_dim = spec.n_embd // spec.n_head
        self.n_embd = spec.n_embd
        self.nsa_block_size = spec.nsa_block_size
        self.nsa_top_k = spec.nsa_top_k
        self.nsa_window_size = spec.nsa_window_size
        self.q_proj = nn.Linear(spec.n_embd, spec.n_embd, bias=spec.bias)
        self.k_proj = nn.Linear(spec.n_embd, spec.n_embd, bias=spec.bias)
        self.v_proj = nn.Linear(spec.n_embd, spec.n_embd, bias=spec.bias)
        self.c_proj = nn.Linear(spec.n_embd, spec.n_embd, bias=spec.bias)
        self.compress_k = nn.Linear(self.head_dim * self.nsa_block_size, self.head_dim, bias=False)
        self.compress_v = nn.Linear(self.head_dim * self.nsa_block_size, self.head_dim, bias=False)
        self.gate = nn.Linear(spec.n_embd, 3 * spec.n_head, bias=False)
        self.rope = (RopeTable(self.head_dim, spec.rope_theta, spec.rope_scaling_type, spec.rope_scaling_factor,
                               spec.block_size) if spec.use_rope else None)
        self.attn_dropout = nn.Dropout(spec.dropout)
        self.resid_dropout = nn.Dropout(spec.dropout)
        self.scale = 1.0 / math.sqrt(self.head_dim)

    def _compressed(self, q, k, v):
        B, H, T, D = k.shape
        bs = self.nsa_block_size
        pad = (-T) % bs
        if pad:
            k = F.pad(k, (0, 0, 0, pad))
            v = F.pad(v, (0, 0, 0, pad))
        nb = k.shape[2] // bs
        kc = self.compress_k(k.reshape(B, H, nb, bs * D))
        vc = self.compress_v(v.reshape(B, H, nb, bs * D))
        s = (q @ kc.transpose(-2, -1)) * self.scale
        mask = torch.triu(torch.ones(T, nb, dtype=torch.bool, device=q.device), diagonal=max(1, nb - T + 1))
        s = s.masked_fill(mask, float("-inf"))
        return torch.softmax(s, -1) @ vc

    def _selected(self, q, k, v):
        B, H, T, D = q.shape
        kk = min(self.nsa_top_k, k.shape[2])
        s = (q @ k.transpose(-2, -1)) * self.scale
        s = s.masked_fill(torch.triu(torch.ones(T, k.shape[2], dtype=torch.bool, device=q.device), 1), float("-inf"))
        top_s, top_i = s.topk(kk, dim=-1)
        gi = top_i.unsqueeze(-1).expand(-1, -1, -1, -1, D)
        vs = torch.gather(v.unsqueeze(2).expand(-1, -1, T, -1, -1), 3, gi)
        p = self.attn_dropout(torch.softmax(top_s, -1))
        return (p.unsqueeze(-2) @ vs).squeeze(-2)

    def _window(self, q, k, v):
        T = q.shape[2]
        s = (q @ k.transpose(-2, -1)) * self.scale
        qp = torch.arange(T, device=q.device)[:, None]
        kp = torch.arange(k.shape[2], device=q.device)[None, :]
        s = s.masked_fill(~((kp <= qp) & (qp - kp < self.nsa_window_size)), float("-inf"))
        return self.attn_dropout(torch.softmax(s, -1)) @ v

    def forward(self, x: torch.Tensor, past_kv: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, positions=None):
        B, T, C = x.shape
        q = self.q_proj(x).view(B, T, self.n_head, self.head_dim).transpose(1, 2)
        k = self.k_proj(x).view(B, T, self.n_head, self.head_dim).transpose(1, 2)
        v = self.v_proj(x).view(B, T, self.n_head, self.head_dim).transpose(1, 2)
        if self.rope is not None:
            q, k = apply_rope(q, self.rope), apply_rope(k, self.rope)
        present = (k, v)
        if past_kv is not None:
            k = torch.cat([past_kv[0], k], 2)
            v = torch.cat([past_kv[1], v], 2)
        gates = torch.softmax(self.gate(x).view(B, T, 3, self.n_head), dim=2).permute(0, 3, 1, 2)
        y = (gates[..., 0:1] * self._compressed(q, k, v) + gates[..., 1:2] * self._selected(q, k, v)
             + gates[..., 2:3] * self._window(q, k, v))
        y = y.transpose(1, 2).reshape(B, T, C)
        return self.resid_dropout(self.c_proj(y)), present
