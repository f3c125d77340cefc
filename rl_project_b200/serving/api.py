"""Transport-independent router of the OpenAI-compatible API.

``Router.handle(method, path, body)`` returns ``(status, dict)`` for JSON and
``(status, iterator of SSE lines)`` for streams, so unit tests and the HTTP
server exercise the same object.  Routes, status mapping (400 invalid request,
503 backend unavailable, 500 other, 404 unknown route) and the ``route_fn``
hook (request id, requested model) -> backend name follow
``src/forgeline/serving/api.py:34-142``.  Latencies are kept in a bounded ring.
"""

from __future__ import annotations

import json
import threading
import time
from collections import deque
from typing import Any, Callable, Dict, Iterator, Optional, Tuple, Union

from rl_project_b200.core.errors import BackendUnavailableError, ServingError
from rl_project_b200.observability.events import Event
from rl_project_b200.observability.logging import get_logger
from rl_project_b200.observability.metrics import MetricsSink, NoOpMetricsSink
from rl_project_b200.serving.backends import Backend
from rl_project_b200.serving.schemas import (ChatCompletionRequest, CompletionRequest, chat_chunk, chat_response,
                                             completion_chunk, completion_response, error_response, new_request_id)

log = get_logger("forgeline.serving")

Response = Tuple[int, Union[Dict[str, Any], Iterator[str]]]

# exception type -> (HTTP status, error code); first match wins (BackendUnavailableError is a ServingError)
_ERRORS = ((BackendUnavailableError, (503, "backend_unavailable")), (ServingError, (400, "invalid_request_error")))


def _percentile(sorted_vals, q: float) -> float:
    if not sorted_vals:
        return 0.0
    return sorted_vals[min(len(sorted_vals) - 1, int(len(sorted_vals) * q))]


class Router:
    def __init__(self, backends: Dict[str, Backend], default_model: str,
                 route_fn: Optional[Callable[[str, Optional[str]], str]] = None,
                 metrics: Optional[MetricsSink] = None, owner: str = "forgeline", latency_window: int = 1000):
        if default_model not in backends:
            raise ServingError(f"default model {default_model!r} is not a registered backend")
        self.backends = dict(backends)
        self.default_model = default_model
        self.route_fn = route_fn
        self.metrics = metrics or NoOpMetricsSink()
        self.owner = owner
        self.requests_total = 0
        self.errors_total = 0
        self.latencies: deque = deque(maxlen=latency_window)
        self._lock = threading.Lock()

    def handle(self, method: str, path: str, body: Optional[Dict[str, Any]] = None) -> Response:
        routes = {("GET", "/health"): lambda: (200, self.health()),
                  ("GET", "/v1/models"): lambda: (200, self.models()),
                  ("GET", "/metrics"): lambda: (200, self.metrics_summary()),
                  ("POST", "/v1/completions"): lambda: self.completions(body or {}),
                  ("POST", "/v1/chat/completions"): lambda: self.chat_completions(body or {})}
        fn = routes.get((method, path))
        if fn is None:
            return 404, error_response(f"no route for {method} {path}", "not_found", 404)
        try:
            return fn()
        except Exception as exc:  # noqa: BLE001 - every failure becomes a JSON error response
            status, code = next((sc for kind, sc in _ERRORS if isinstance(exc, kind)), (500, "server_error"))
            self._error(exc)
            msg = str(getattr(exc, "message", exc)) if status != 500 else f"{type(exc).__name__}: {exc}"
            return status, error_response(msg, code, status)

    def _error(self, exc: BaseException) -> None:
        with self._lock:
            self.errors_total += 1
        log.warning("serving_error", error=repr(exc))
        self.metrics.increment("serving/errors")
        self.metrics.event(Event.SERVING_ERROR.value, {"error": repr(exc)})

    # ------------------------------------------------------------ endpoints
    def health(self) -> Dict[str, Any]:
        status = {name: b.healthy() for name, b in self.backends.items()}
        return {"status": "ok" if status.get(self.default_model, False) else "degraded", "backends": status,
                "default_model": self.default_model}

    def models(self) -> Dict[str, Any]:
        return {"object": "list", "data": [{"id": n, "object": "model", "owned_by": self.owner,
                                            "healthy": b.healthy()} for n, b in self.backends.items()]}

    def metrics_summary(self) -> Dict[str, Any]:
        with self._lock:
            lat = sorted(self.latencies)
            return {"requests_total": self.requests_total, "errors_total": self.errors_total,
                    "latency_p50_s": _percentile(lat, 0.5), "latency_p95_s": _percentile(lat, 0.95),
                    "backends": list(self.backends)}

    def _select_backend(self, request_id: str, requested: Optional[str]) -> Tuple[str, Backend]:
        name = self.route_fn(request_id, requested) if self.route_fn else (requested or self.default_model)
        if name not in self.backends:
            raise ServingError(f"unknown model {name!r}; available: {sorted(self.backends)}")
        backend = self.backends[name]
        if not backend.healthy():
            raise BackendUnavailableError(f"backend {name!r} is unavailable")
        return name, backend

    def _serve(self, req, prompt: str, respond, chunk) -> Response:
        rid = req.request_id or new_request_id()
        name, backend = self._select_backend(rid, req.model)
        with self._lock:
            self.requests_total += 1
        t0 = time.perf_counter()
        if req.stream:
            pieces = backend.stream(prompt, req.sampling(), rid, stop=req.stop)
            return 200, self._sse(pieces, lambda t, fr: chunk(rid, name, t, fr), t0, name)
        res = backend.complete(prompt, req.sampling(), rid, stop=req.stop)
        self._record(t0, res.completion_tokens, name)
        return 200, respond(rid, name, res.text, res.prompt_tokens, res.completion_tokens, res.finish_reason, name)

    def completions(self, body: Dict[str, Any]) -> Response:
        req = CompletionRequest.from_dict(body)
        return self._serve(req, req.prompt, completion_response, completion_chunk)

    def chat_completions(self, body: Dict[str, Any]) -> Response:
        req = ChatCompletionRequest.from_dict(body)
        return self._serve(req, req.to_prompt(), chat_response, chat_chunk)

    def _sse(self, pieces: Iterator[str], make, t0: float, backend: str) -> Iterator[str]:
        n = 0
        for text in pieces:
            n += 1
            yield f"data: {json.dumps(make(text, None))}\n\n"
        yield f"data: {json.dumps(make('', 'stop'))}\n\n"
        yield "data: [DONE]\n\n"
        self._record(t0, n, backend)

    def _record(self, t0: float, tokens: int, backend: str) -> None:
        latency = time.perf_counter() - t0
        with self._lock:
            self.latencies.append(latency)
        self.metrics.log({"serving/latency_s": latency, "serving/completion_tokens": float(tokens)})
        self.metrics.increment("serving/requests")
        self.metrics.event(Event.SERVING_REQUEST.value, {"backend": backend, "latency_s": latency, "tokens": tokens})
