"""Transformer block and multi-token-prediction module
(``src/forgeline/models/transformer/block.py:19-67``).

``TransformerBlock.forward(x, past_kv)`` keeps the reference signature.
``forward_fused(x, pending)`` is the training/prefill path: the residual add
left over from the previous block (``pending``) is folded into this block's
``ln_1`` kernel and the attention residual into ``ln_2``, so every residual
add costs no extra pass over the activations.
"""

from __future__ import annotations

from typing import Any, Optional, Tuple

import torch
import torch.nn as nn

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.models.attention.causal import CausalSelfAttention
from rl_project_b200.models.attention.latent import MultiHeadLatentAttention
from rl_project_b200.models.attention.sparse import NativeSparseAttention
from rl_project_b200.models.moe.layer import MoELayer
from rl_project_b200.models.transformer.feedforward import make_ffn
from rl_project_b200.models.transformer.norm import RMSNorm
from rl_project_b200.ops.norm import add_rms_norm, rms_norm


def build_attention(spec: ModelSpec, layer_id: int = 0) -> nn.Module:
    if spec.use_mla:
        return MultiHeadLatentAttention(spec)
    if spec.use_nsa:
        return NativeSparseAttention(spec)
    return CausalSelfAttention(spec, layer_id=layer_id)


def build_dense_ffn(spec: ModelSpec) -> nn.Module:
    return make_ffn(spec)


class TransformerBlock(nn.Module):
    def __init__(self, layer_id: int, spec: ModelSpec):
        super().__init__()
        self.layer_id = layer_id
        self.ln_1 = RMSNorm(spec.n_embd)
        self.ln_2 = RMSNorm(spec.n_embd)
        self.attn = build_attention(spec, layer_id)
        self.use_moe = bool(spec.use_moe and layer_id >= spec.n_dense_layers)
        self.ffn = MoELayer(spec) if self.use_moe else build_dense_ffn(spec)

    def forward(self, x: torch.Tensor, past_kv: Optional[Any] = None, positions=None, *,
                pending: Optional[torch.Tensor] = None, fused: bool = False):
        if fused:
            return self.forward_fused(x, pending)
        a, present = self.attn(self.ln_1(x), past_kv=past_kv, positions=positions)
        x, h = add_rms_norm(x, a, self.ln_2.weight, self.ln_2.eps)
        return x + self.ffn(h), present

    def forward_paged(self, x: torch.Tensor, kv, meta) -> torch.Tensor:
        """Decode step over the paged KV pools (``CausalSelfAttention`` layers only)."""
        a = self.attn.forward_paged(self.ln_1(x), kv, meta)
        x, h = add_rms_norm(x, a, self.ln_2.weight, self.ln_2.eps)
        return x + self.ffn(h)

    def forward_fused(self, x: torch.Tensor, pending: Optional[torch.Tensor]) -> Tuple[torch.Tensor, torch.Tensor]:
        """Returns ``(x, f)`` with the block output equal to ``x + f`` (add left pending).

        Call it as ``block(x, pending=p, fused=True)`` so module hooks (FSDP gathers) run."""
        if pending is None:
            h = rms_norm(x, self.ln_1.weight, self.ln_1.eps)
        else:
            x, h = add_rms_norm(x, pending, self.ln_1.weight, self.ln_1.eps)
        a, _ = self.attn(h)
        x, h = add_rms_norm(x, a, self.ln_2.weight, self.ln_2.eps)
        return x, self.ffn(h)


class MTPModule(nn.Module):
    """One extra prediction depth: ``norm(proj(h) + emb(next))`` -> attention -> FFN."""

    def __init__(self, spec: ModelSpec):
        super().__init__()
        self.proj = nn.Linear(spec.n_embd, spec.n_embd, bias=False)
        self.norm = RMSNorm(spec.n_embd)
        self.attn_norm = RMSNorm(spec.n_embd)
        self.attn = MultiHeadLatentAttention(spec) if spec.use_mla else CausalSelfAttention(spec)
        self.ffn_norm = RMSNorm(spec.n_embd)
        self.ffn = build_dense_ffn(spec)

    def forward(self, h: torch.Tensor, target_emb: torch.Tensor) -> torch.Tensor:
        c = self.norm(self.proj(h) + target_emb)
        a, _ = self.attn(self.attn_norm(c))
        c = c + a
        return c + self.ffn(self.ffn_norm(c))
