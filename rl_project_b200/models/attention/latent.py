"""Multi-head latent attention (``src/forgeline/models/attention/latent.py:17-128``).

Low-rank KV (``wkv_a -> [c_kv | k_rope]``, ``kv_norm``, ``wkv_b``), optional
q-LoRA (``wq_a``/``q_norm``/``wq_b``), decoupled RoPE on ``qk_rope_head_dim``.
Cache ``(c_kv [B, T, r], k_rope [B, 1, T, d_r])``.  Training / prefill use the
decompressed ("naive") path (cuDNN SDPA, or the own d_qk 192 / d_v 128 forward
kernel for inference prefill); single-token eval decode uses the absorbed path:
multi-query attention over one shared ``r + d_r``-wide key in the latent space.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.models.transformer.norm import RMSNorm
from rl_project_b200.ops.attention import attention_reference
from rl_project_b200.ops.rope import RopeTable, apply_rope

LatentCache = Tuple[torch.Tensor, torch.Tensor]


class MultiHeadLatentAttention(nn.Module):
    def __init__(self, spec: ModelSpec):
        super().__init__()
        self.n_heads = spec.n_head
        self.dim = spec.n_embd
        self.kv_lora_rank = spec.kv_lora_rank
        self.q_lora_rank = spec.q_lora_rank
        self.qk_nope_head_dim = spec.qk_nope_head_dim
        self.qk_rope_head_dim = spec.qk_rope_head_dim
        self.qk_head_dim = spec.qk_nope_head_dim + spec.qk_rope_head_dim
        self.v_head_dim = spec.v_head_dim
        self.attn_logit_cap = spec.attn_logit_cap
        if self.q_lora_rank == 0:
            self.wq = nn.Linear(self.dim, self.n_heads * self.qk_head_dim, bias=False)
        else:
            self.wq_a = nn.Linear(self.dim, self.q_lora_rank, bias=False)
            self.q_norm = RMSNorm(self.q_lora_rank)
            self.wq_b = nn.Linear(self.q_lora_rank, self.n_heads * self.qk_head_dim, bias=False)
        self.wkv_a = nn.Linear(self.dim, self.kv_lora_rank + self.qk_rope_head_dim, bias=False)
        self.kv_norm = RMSNorm(self.kv_lora_rank)
        self.wkv_b = nn.Linear(self.kv_lora_rank, self.n_heads * (self.qk_nope_head_dim + self.v_head_dim), bias=False)
        self.wo = nn.Linear(self.n_heads * self.v_head_dim, self.dim, bias=False)
        self.rope = RopeTable(self.qk_rope_head_dim, spec.rope_theta, spec.rope_scaling_type,
                              spec.rope_scaling_factor, spec.block_size)
        self.softmax_scale = self.qk_head_dim ** -0.5
        self.attn_dropout = nn.Dropout(spec.dropout)
        self.resid_dropout = nn.Dropout(spec.dropout)

    def _naive(self, q_nope, q_rope, kv_latent, k_rope, T):
        B = q_nope.shape[0]
        kv = self.wkv_b(kv_latent).view(B, -1, self.n_heads, self.qk_nope_head_dim + self.v_head_dim)
        k_nope, v = kv.split([self.qk_nope_head_dim, self.v_head_dim], dim=-1)
        k = torch.cat([k_nope.transpose(1, 2), k_rope.expand(-1, self.n_heads, -1, -1)], dim=-1)
        q = torch.cat([q_nope.transpose(1, 2), q_rope], dim=-1)
        v = v.transpose(1, 2)
        if q.is_cuda and self.attn_logit_cap == 0 and T == k.shape[2] and not torch.is_grad_enabled():
            from rl_project_b200.ops import attention as A

            if A._ATTN == "tcgen05" and q.dtype == torch.bfloat16 and (q.shape[-1], v.shape[-1]) in A.FMHA_SHAPES:
                return A.fmha_forward(q, k, v, True, self.softmax_scale)[0]  # own kernel (prefill; forward only)
        if q.is_cuda and self.attn_logit_cap == 0 and T == k.shape[2]:
            import torch.nn.functional as F

            y = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=self.softmax_scale,
                                               dropout_p=self.attn_dropout.p if self.training else 0.0)
            return y
        return attention_reference(q, k, v, softcap=self.attn_logit_cap, scale=self.softmax_scale,
                                   q_offset=k.shape[2] - T)

    def _absorbed(self, q_nope, q_rope, kv_latent, k_rope, T):
        """Attention in the latent space, as multi-query attention over ONE shared key of width
        ``kv_lora_rank + qk_rope_head_dim``: each head's no-RoPE query is mapped into the latent space by its
        slice of ``wkv_b`` and concatenated with its RoPE query, the cached ``[latent | k_rope]`` rows are the
        keys, the latent rows the values, and ``wkv_b``'s value slice maps the result back per head."""
        S = kv_latent.shape[1]
        w = self.wkv_b.weight.view(self.n_heads, self.qk_nope_head_dim + self.v_head_dim, self.kv_lora_rank)
        w_k, w_v = w.split([self.qk_nope_head_dim, self.v_head_dim], dim=1)
        q_cat = torch.cat([torch.einsum("bthn,hnl->bhtl", q_nope, w_k), q_rope], dim=-1)  # [B, H, T, r + d_r]
        k_cat = torch.cat([kv_latent, k_rope[:, 0]], dim=-1).unsqueeze(1)  # [B, 1, S, r + d_r]
        scores = (q_cat @ k_cat.transpose(-2, -1)) * self.softmax_scale
        if self.attn_logit_cap > 0:
            scores = torch.tanh(scores / self.attn_logit_cap) * self.attn_logit_cap
        if T > 1:
            future = torch.arange(S, device=scores.device)[None, :] > torch.arange(S - T, S, device=scores.device)[:, None]
            scores = scores.masked_fill(future, float("-inf"))
        p = scores.float().softmax(-1).type_as(q_nope)
        return torch.einsum("bhtl,hvl->bhtv", p @ kv_latent.unsqueeze(1), w_v)

    def forward(self, x: torch.Tensor, past_kv: Optional[LatentCache] = None, positions=None):
        B, T, _ = x.shape
        q = self.wq(x) if self.q_lora_rank == 0 else self.wq_b(self.q_norm(self.wq_a(x)))
        q = q.view(B, T, self.n_heads, self.qk_head_dim)
        q_nope, q_rope = q.split([self.qk_nope_head_dim, self.qk_rope_head_dim], dim=-1)
        kv_latent, k_rope = self.wkv_a(x).split([self.kv_lora_rank, self.qk_rope_head_dim], dim=-1)
        kv_latent = self.kv_norm(kv_latent)
        offset = past_kv[0].shape[1] if past_kv is not None else 0
        q_rope = apply_rope(q_rope.transpose(1, 2), self.rope, offset)
        k_rope = apply_rope(k_rope.unsqueeze(1), self.rope, offset)
        if past_kv is not None:
            kv_latent = torch.cat([past_kv[0], kv_latent], dim=1)
            k_rope = torch.cat([past_kv[1], k_rope], dim=2)
        present = (kv_latent, k_rope)
        if (not self.training) and T == 1:
            y = self._absorbed(q_nope, q_rope, kv_latent, k_rope, T)
        else:
            y = self._naive(q_nope, q_rope, kv_latent, k_rope, T)
        y = y.transpose(1, 2).reshape(B, T, self.n_heads * self.v_head_dim)
        return self.resid_dropout(self.wo(y)), present
