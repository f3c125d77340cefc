"""Inference: request life cycle, paged KV cache (block accounting + device pool),
continuous-batching scheduler and engine, text generation."""

from rl_project_b200.inference.engine import InferenceEngine
from rl_project_b200.inference.generation import generate_text
from rl_project_b200.inference.paged_memory import OutOfBlocksError, PagedBlockAllocator, PagedKVCache
from rl_project_b200.inference.requests import GenerationRequest, RequestStatus, SamplingParams
from rl_project_b200.inference.scheduler import Scheduler

__all__ = ["InferenceEngine", "generate_text", "OutOfBlocksError", "PagedBlockAllocator", "PagedKVCache",
           "GenerationRequest", "RequestStatus", "SamplingParams", "Scheduler"]
