"""Native sparse attention (the branches and gate of ``src/forgeline/models/attention/sparse.py``):
compressed-block, top-k selected and sliding-window attention mixed by a learned per-head softmax gate.
Like the reference, no cached decode.

The selected and windowed branches attend over the same keys and values, so they share one score matrix,
express their key sets as masks over it, and combine as ``(g_sel P_sel + g_win P_win) @ V`` -- one
probability-by-value product instead of a gathered ``[B, H, T, k, D]`` value tensor plus a second product.
"""

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
        """Attention over block summaries: every ``nsa_block_size`` keys / values compressed by a linear map."""
        B, H, T, D = k.shape
        bs = self.nsa_block_size
        pad = (-T) % bs
        if pad:
            k, v = F.pad(k, (0, 0, 0, pad)), F.pad(v, (0, 0, 0, pad))
        nb = k.shape[2] // bs
        kc = self.compress_k(k.reshape(B, H, nb, bs * D))
        vc = self.compress_v(v.reshape(B, H, nb, bs * D))
        s = (q @ kc.transpose(-2, -1)) * self.scale
        hidden = torch.triu(torch.ones(T, nb, dtype=torch.bool, device=q.device), diagonal=max(1, nb - T + 1))
        return torch.softmax(s.masked_fill(hidden, float("-inf")), -1) @ vc

    def _fine_probs(self, q, k):
        """The selected and windowed branches' attention probabilities ``[B, H, T, S]``, both from ONE score
        matrix: selection keeps each query's ``nsa_top_k`` best causal keys (a softmax over them equals a
        softmax over the row with every other key masked), the window keeps the last ``nsa_window_size``."""
        T, S = q.shape[2], k.shape[2]
        scores = (q @ k.transpose(-2, -1)) * self.scale
        qp = torch.arange(T, device=q.device)[:, None]
        kp = torch.arange(S, device=q.device)[None, :]
        causal = kp <= qp
        neg = float("-inf")
        s_causal = scores.masked_fill(~causal, neg)
        top = s_causal.topk(min(self.nsa_top_k, S), dim=-1).indices
        chosen = torch.zeros_like(s_causal, dtype=torch.bool).scatter_(-1, top, True)
        p_sel = torch.softmax(s_causal.masked_fill(~chosen, neg), -1)
        p_win = torch.softmax(scores.masked_fill(~(causal & (qp - kp < self.nsa_window_size)), neg), -1)
        return self.attn_dropout(p_sel), self.attn_dropout(p_win)

    def forward(self, x: torch.Tensor, past_kv: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, positions=None):
        B, T, C = x.shape
        heads = lambda t: t.view(B, T, self.n_head, self.head_dim).transpose(1, 2)  # noqa: E731
        q, k, v = heads(self.q_proj(x)), heads(self.k_proj(x)), heads(self.v_proj(x))
        if self.rope is not None:
            q, k = apply_rope(q, self.rope), apply_rope(k, self.rope)
        present = (k, v)
        if past_kv is not None:
            k = torch.cat([past_kv[0], k], 2)
            v = torch.cat([past_kv[1], v], 2)
        g = torch.softmax(self.gate(x).view(B, T, 3, self.n_head), dim=2).permute(0, 3, 1, 2)  # [B, H, T, 3]
        p_sel, p_win = self._fine_probs(q, k)
        # the two fine branches share their values: one (weighted probabilities) @ v product for both
        fine = (g[..., 1:2] * p_sel + g[..., 2:3] * p_win) @ v
        y = g[..., 0:1] * self._compressed(q, k, v) + fine
        return self.resid_dropout(self.c_proj(y.transpose(1, 2).reshape(B, T, C))), present
