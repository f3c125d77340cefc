"""OpenAI-compatible serving: schemas, backends, router and HTTP server."""

from rl_project_b200.serving.api import Router
from rl_project_b200.serving.backends import CompletionResult, EchoBackend, EngineBackend
from rl_project_b200.serving.schemas import ChatCompletionRequest, CompletionRequest
from rl_project_b200.serving.server import ServingServer

__all__ = ["Router", "CompletionResult", "EchoBackend", "EngineBackend", "ChatCompletionRequest",
           "CompletionRequest", "ServingServer"]
