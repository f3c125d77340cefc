"""Attention variants: grouped-query causal, multi-head latent, native sparse."""

from rl_project_b200.models.attention.causal import CausalSelfAttention
from rl_project_b200.models.attention.latent import MultiHeadLatentAttention
from rl_project_b200.models.attention.rotary import (
    RotaryEmbedding,
    apply_rotary_pos_emb,
    apply_rotary_pos_emb_pair,
)
from rl_project_b200.models.attention.sparse import NativeSparseAttention
