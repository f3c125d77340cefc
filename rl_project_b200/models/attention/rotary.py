"""RoPE module API (``src/forgeline/models/attention/rotary.py``) over ``ops.rope.RopeTable``."""

from __future__ import annotations

import torch
import torch.nn as nn

from rl_project_b200.ops.rope import RopeTable, apply_rope_reference


class RotaryEmbedding(nn.Module):
    """``forward(seq_len, offset)`` returns full-width ``(cos, sin)`` ``[T, dim]`` like the reference."""

    def __init__(self, dim: int, max_seq_len: int = 8192, base: float = 10000.0, scaling_type: str = "none",
                 scaling_factor: float = 1.0):
        super().__init__()
        self.dim = dim
        self.table = RopeTable(dim, base, scaling_type, scaling_factor, max_seq_len)
        self.register_buffer("inv_freq", self.table.inv_freq.clone(), persistent=False)

    def forward(self, seq_len: int, offset: int = 0):
        cos, sin = self.table.tables(offset + seq_len, self.inv_freq.device)
        c, s = cos[offset:offset + seq_len], sin[offset:offset + seq_len]
        return torch.cat([c, c], -1), torch.cat([s, s], -1)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    a, b = x.chunk(2, dim=-1)
    return torch.cat((-b, a), dim=-1)


def apply_rotary_pos_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """``x [B, H, T, D]`` with full-width ``cos/sin [T, D]``."""
    half = x.shape[-1] // 2
    return apply_rope_reference(x, cos[..., :half], sin[..., :half])


def apply_rotary_pos_emb_pair(q, k, cos, sin):
    return apply_rotary_pos_emb(q, cos, sin), apply_rotary_pos_emb(k, cos, sin)
