"""Decoder-only transformer."""

from rl_project_b200.models.transformer.block import MTPModule, TransformerBlock
from rl_project_b200.models.transformer.feedforward import GELUFeedForward, SwiGLUFeedForward, make_ffn
from rl_project_b200.models.transformer.model import TransformerLM
from rl_project_b200.models.transformer.norm import RMSNorm
