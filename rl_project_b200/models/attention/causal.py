"""Grouped-query causal self-attention with KV cache, sliding window and logit cap.

Behaviour and parameter names follow ``src/forgeline/models/attention/causal.py:18-134``
(``q_proj``/``k_proj``/``v_proj``/``c_proj``; window on every layer or on odd
layers only; tanh soft-cap; ``(k, v)`` cache ``[B, Hkv, T, D]``).  The three
projections run as ONE GEMM over the concatenated weight and RoPE is fused
with the head split (csrc/rope.cu).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn as nn

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.ops import gemm
from rl_project_b200.ops.attention import attention_reference, causal_attention
from rl_project_b200.ops.linear import linear
from rl_project_b200.ops.paged_attention import paged_decode, paged_write
from rl_project_b200.ops.rope import RopeTable, rope_split_qkv

KVCache = Tuple[torch.Tensor, torch.Tensor]


@dataclass
class PagedDecodeMeta:
    """Per-step addressing of a batch of sequences decoding one token each.

    ``positions [B, 1]`` is each new token's position (= cached tokens before
    it); its K/V go to block ``slot_block[b]``, offset ``slot_off[b]``; attention
    then covers ``ctx_lens[b] = positions[b] + 1`` tokens through
    ``block_tables [B, max_blocks]``.  All int32 on the model's device.
    """

    positions: torch.Tensor
    max_pos: int
    block_tables: torch.Tensor
    ctx_lens: torch.Tensor
    slot_block: torch.Tensor
    slot_off: torch.Tensor
    split_tokens: int = 0


def layer_window(spec: ModelSpec, layer_id: int) -> int:
    if spec.alternating_layers:
        return spec.sliding_window if layer_id % 2 == 1 else 0
    return spec.sliding_window if spec.sliding_window > 0 else 0


class CausalSelfAttention(nn.Module):
    def __init__(self, spec: ModelSpec, layer_id: int = 0):
        super().__init__()
        self.n_head = spec.n_head
        self.n_kv_head = spec.n_kv_head
        self.n_embd = spec.n_embd
        self.head_dim = spec.n_embd // spec.n_head
        self.n_rep = spec.n_head // spec.n_kv_head
        self.dropout_rate = spec.dropout
        self.use_rope = spec.use_rope
        self.attn_logit_cap = spec.attn_logit_cap
        self.window_size = layer_window(spec, layer_id)
        self.q_proj = nn.Linear(spec.n_embd, spec.n_head * self.head_dim, bias=spec.bias)
        self.k_proj = nn.Linear(spec.n_embd, spec.n_kv_head * self.head_dim, bias=spec.bias)
        self.v_proj = nn.Linear(spec.n_embd, spec.n_kv_head * self.head_dim, bias=spec.bias)
        self.c_proj = nn.Linear(spec.n_embd, spec.n_embd, bias=spec.bias)
        self.resid_dropout = nn.Dropout(spec.dropout)
        self.rope = RopeTable(self.head_dim, spec.rope_theta, spec.rope_scaling_type, spec.rope_scaling_factor,
                              spec.block_size)
        self.tp_group = None  # set by tensor parallelism (heads then divided over the group)

    def _qkv(self, x: torch.Tensor) -> torch.Tensor:
        """q|k|v projections as one GEMM; under tensor parallelism ``x`` is the replicated block
        input and the input-gradient all-reduce belongs to this projection."""
        mods = (self.q_proj, self.k_proj, self.v_proj)
        fused = all(type(m) is nn.Linear for m in mods)
        if self.tp_group is not None:
            from rl_project_b200.parallel.tensor_parallel import column_parallel_in, copy_to_tp
        if fused:
            w = torch.cat([m.weight for m in mods], 0)
            b = torch.cat([m.bias for m in mods], 0) if self.q_proj.bias is not None else None
            if self.tp_group is not None:
                return column_parallel_in(x, w, b, self.tp_group)
            return linear(x, w, b)
        if self.tp_group is not None:
            x = copy_to_tp(x, self.tp_group)
        return torch.cat([m(x) for m in mods], dim=-1)

    def _out(self, y: torch.Tensor) -> torch.Tensor:
        if self.tp_group is not None:
            from rl_project_b200.parallel.tensor_parallel import row_parallel_out

            y = row_parallel_out(y, self.c_proj, self.tp_group)
        elif type(self.c_proj) is nn.Linear:
            y = linear(y, self.c_proj.weight, self.c_proj.bias)
        else:
            y = self.c_proj(y)
        return self.resid_dropout(y)

    def _rope_qkv_fused(self, x: torch.Tensor, offset: int, positions: Optional[torch.Tensor]):
        """q, k, v from one GEMM whose epilogue applies RoPE and splits the heads, when the own GEMM runs the
        forward projections; None otherwise."""
        mods = (self.q_proj, self.k_proj, self.v_proj)
        if not (self.use_rope and self.tp_group is None and x.is_cuda and x.dtype == torch.bfloat16
                and positions is None and all(type(m) is nn.Linear and m.bias is None for m in mods)):
            return None
        rows = x.shape[0] * x.shape[1]
        if not (gemm.enabled() and gemm.fills_gpu(rows, sum(m.weight.shape[0] for m in mods), 512,
                                                   x.device.index or 0)):
            return None  # decided before concatenating the weights
        w = torch.cat([m.weight for m in mods], 0)
        if not gemm.rope_qkv_fusable(x.reshape(-1, x.shape[-1]), w, self.n_head, self.n_kv_head, self.head_dim):
            return None
        cos, sin = self.rope.tables(offset + x.shape[1], x.device)
        return gemm.linear_rope_qkv(x, w, cos, sin, None, self.n_head, self.n_kv_head, self.head_dim, offset)

    def forward(self, x: torch.Tensor, past_kv: Optional[KVCache] = None, positions: Optional[torch.Tensor] = None):
        B, T, C = x.shape
        offset = past_kv[0].shape[2] if past_kv is not None else 0
        # q/k/v come out token-major [B, T, H, D]; attention reads them through [B, H, T, D]
        # views so its output is already in the [B, T, H*D] layout the output projection wants
        fused = self._rope_qkv_fused(x, offset, positions)
        if fused is not None:
            q, k, v = fused
        else:
            q, k, v = rope_split_qkv(self._qkv(x), self.rope, self.n_head, self.n_kv_head, self.head_dim,
                                     offset=offset, positions=positions, rotate=self.use_rope, heads_major=False)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if past_kv is not None:
            k = torch.cat([past_kv[0], k], dim=2)
            v = torch.cat([past_kv[1], v], dim=2)
        present = (k, v)
        drop = self.dropout_rate if self.training else 0.0
        if past_kv is None:
            y = causal_attention(q, k, v, window=self.window_size, softcap=self.attn_logit_cap, dropout_p=drop)
        else:
            y = attention_reference(q, k, v, window=self.window_size, softcap=self.attn_logit_cap,
                                    q_offset=k.shape[2] - T)
        y = y.transpose(1, 2).reshape(B, T, self.n_head * self.head_dim)
        return self._out(y), present

    def forward_paged(self, x: torch.Tensor, kv: KVCache, meta: PagedDecodeMeta) -> torch.Tensor:
        """One new token per sequence (``x [B, 1, C]``) against this layer's paged K/V pools."""
        B = x.shape[0]
        qkv = self._qkv(x)
        q, k, v = rope_split_qkv(qkv, self.rope, self.n_head, self.n_kv_head, self.head_dim,
                                 positions=meta.positions, rotate=self.use_rope, heads_major=False,
                                 max_pos=meta.max_pos)
        paged_write(k[:, 0], v[:, 0], kv[0], kv[1], meta.slot_block, meta.slot_off)
        y = paged_decode(q[:, 0], kv[0], kv[1], meta.block_tables, meta.ctx_lens, 1.0 / math.sqrt(self.head_dim),
                         self.attn_logit_cap, self.window_size, meta.split_tokens)
        return self._out(y.reshape(B, 1, self.n_head * self.head_dim))
