"""Sampling and speculative decoding."""

from rl_project_b200.models.generation.sampling import apply_sampling_filters, generate_tokens, sample_from_logits
