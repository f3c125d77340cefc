"""HTTP front end of the OpenAI-compatible router, on the shared asyncio server core (``serving/http.py``).

The router and its backends block on the GPU engine, so they run in the core's thread pool; a streamed
completion is pulled from the backend one piece at a time there and each Server-Sent-Events line is written
as soon as it exists.  Routes, status codes and the wire format are the router's (``serving/api.py``).
"""

from __future__ import annotations

import json
from typing import Dict, Tuple

from rl_project_b200.serving.api import Router
from rl_project_b200.serving.http import MAX_BODY_BYTES, AsyncHTTPServer, Payload  # noqa: F401
from rl_project_b200.serving.schemas import error_response


def _error_body(status: int, message: str) -> bytes:
    code = "server_error" if status >= 500 else "invalid_request_error"
    return json.dumps(error_response(message, code, status)).encode()


class ServingServer:
    """``start()`` serves on a background thread, ``serve_forever()`` on the caller's; ``port`` is the bound
    port (``port=0`` picks a free one); ``stop()`` shuts the server down."""

    def __init__(self, router: Router, host: str = "127.0.0.1", port: int = 8000, workers: int = 8):
        self.router = router
        self._http = AsyncHTTPServer(self._app, host, port, workers, on_bad_request=_error_body)

    def _app(self, method: str, target: str, headers: Dict[str, str], body: bytes) -> Tuple[int, str, Payload]:
        doc = None
        if method == "POST":
            try:
                doc = json.loads(body) if body else {}
            except json.JSONDecodeError:
                return 400, "application/json", _error_body(400, "invalid JSON body")
        status, payload = self.router.handle(method, target.split("?")[0], doc)
        if isinstance(payload, dict):
            return status, "application/json", json.dumps(payload).encode()
        return status, "text/event-stream", payload

    @property
    def port(self) -> int:
        return self._http.port

    def start(self) -> None:
        self._http.start("forgeline-serve")

    def serve_forever(self) -> None:
        self._http.serve_forever()

    def stop(self) -> None:
        self._http.stop()
