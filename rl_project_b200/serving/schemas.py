"""OpenAI-compatible request / response bodies.

The JSON field names and response shapes are the OpenAI completions / chat
completions wire format, which the reference also speaks
(``src/forgeline/serving/schemas.py:15-141``): clients written for either
server work with this one.  Requests are validated into dataclasses;
validation errors raise ``ServingError`` (HTTP 400 at the router).
"""

from __future__ import annotations

import time
import uuid
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

from rl_project_b200.core.errors import ServingError
from rl_project_b200.inference.requests import SamplingParams

CHAT_ROLES = ("system", "user", "assistant", "tool")


def _stop_list(value: Any) -> List[str]:
    if value is None:
        return []
    if isinstance(value, str):
        return [value]
    if isinstance(value, list) and all(isinstance(s, str) for s in value):
        return list(value)
    raise ServingError("'stop' must be a string or a list of strings")


def _common(d: Dict[str, Any]) -> Dict[str, Any]:
    try:
        return {"model": d.get("model"), "max_tokens": int(d.get("max_tokens", 64)),
                "temperature": float(d.get("temperature", 0.8)), "top_k": d.get("top_k", 50),
                "top_p": d.get("top_p"), "stream": bool(d.get("stream", False)), "stop": _stop_list(d.get("stop")),
                "user": d.get("user"), "request_id": d.get("request_id")}
    except (TypeError, ValueError) as exc:
        raise ServingError(f"invalid numeric field: {exc}") from exc


@dataclass
class _SamplingFields:
    model: Optional[str] = None
    max_tokens: int = 64
    temperature: float = 0.8
    top_k: Optional[int] = 50
    top_p: Optional[float] = None
    stream: bool = False
    stop: List[str] = field(default_factory=list)
    user: Optional[str] = None
    request_id: Optional[str] = None

    def sampling(self) -> SamplingParams:
        return SamplingParams(max_tokens=self.max_tokens, temperature=self.temperature, top_k=self.top_k,
                              top_p=self.top_p)


@dataclass
class CompletionRequest(_SamplingFields):
    prompt: str = ""

    @classmethod
    def from_dict(cls, d: Any) -> "CompletionRequest":
        if not isinstance(d, dict):
            raise ServingError("request body must be a JSON object")
        prompt = d.get("prompt")
        if isinstance(prompt, list):  # OpenAI allows a batch; one prompt per request here
            prompt = prompt[0] if prompt else ""
        if not isinstance(prompt, str) or not prompt:
            raise ServingError("'prompt' must be a non-empty string")
        req = cls(prompt=prompt, **_common(d))
        req.sampling().validate()
        return req


@dataclass
class ChatMessage:
    role: str
    content: str


@dataclass
class ChatCompletionRequest(_SamplingFields):
    messages: List[ChatMessage] = field(default_factory=list)

    @classmethod
    def from_dict(cls, d: Any) -> "ChatCompletionRequest":
        if not isinstance(d, dict):
            raise ServingError("request body must be a JSON object")
        raw = d.get("messages")
        if not isinstance(raw, list) or not raw:
            raise ServingError("'messages' must be a non-empty list")
        msgs = []
        for m in raw:
            if not isinstance(m, dict) or not isinstance(m.get("content"), str):
                raise ServingError("each message needs a string 'content'")
            role = m.get("role", "user")
            if role not in CHAT_ROLES:
                raise ServingError(f"invalid role {role!r}; expected one of {CHAT_ROLES}")
            msgs.append(ChatMessage(role=role, content=m["content"]))
        req = cls(messages=msgs, **_common(d))
        req.sampling().validate()
        return req

    def to_prompt(self) -> str:
        """Role-tagged transcript ending with an open assistant turn."""
        parts = [f"<|{m.role}|>\n{m.content}\n" for m in self.messages]
        return "".join(parts) + "<|assistant|>\n"


def _usage(prompt_tokens: int, completion_tokens: int) -> Dict[str, int]:
    return {"prompt_tokens": prompt_tokens, "completion_tokens": completion_tokens,
            "total_tokens": prompt_tokens + completion_tokens}


def completion_response(request_id: str, model: str, text: str, prompt_tokens: int, completion_tokens: int,
                        finish_reason: str, backend: Optional[str] = None) -> Dict[str, Any]:
    out: Dict[str, Any] = {"id": f"cmpl-{request_id}", "object": "text_completion", "created": int(time.time()),
                           "model": model,
                           "choices": [{"text": text, "index": 0, "finish_reason": finish_reason, "logprobs": None}],
                           "usage": _usage(prompt_tokens, completion_tokens)}
    if backend:
        out["forgeline"] = {"backend": backend}
    return out


def chat_response(request_id: str, model: str, text: str, prompt_tokens: int, completion_tokens: int,
                  finish_reason: str, backend: Optional[str] = None) -> Dict[str, Any]:
    out: Dict[str, Any] = {"id": f"chatcmpl-{request_id}", "object": "chat.completion", "created": int(time.time()),
                           "model": model,
                           "choices": [{"index": 0, "message": {"role": "assistant", "content": text},
                                        "finish_reason": finish_reason}],
                           "usage": _usage(prompt_tokens, completion_tokens)}
    if backend:
        out["forgeline"] = {"backend": backend}
    return out


def completion_chunk(request_id: str, model: str, text: str, finish_reason: Optional[str] = None) -> Dict[str, Any]:
    return {"id": f"cmpl-{request_id}", "object": "text_completion", "created": int(time.time()), "model": model,
            "choices": [{"text": text, "index": 0, "finish_reason": finish_reason}]}


def chat_chunk(request_id: str, model: str, text: str, finish_reason: Optional[str] = None) -> Dict[str, Any]:
    return {"id": f"chatcmpl-{request_id}", "object": "chat.completion.chunk", "created": int(time.time()),
            "model": model, "choices": [{"index": 0, "delta": {"content": text}, "finish_reason": finish_reason}]}


def error_response(message: str, kind: str = "invalid_request_error", code: int = 400) -> Dict[str, Any]:
    return {"error": {"message": message, "type": kind, "code": code}}


def new_request_id() -> str:
    return uuid.uuid4().hex[:24]
