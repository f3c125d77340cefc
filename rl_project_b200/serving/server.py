"""Standard-library HTTP server for the router (threaded; SSE for streams)."""

from __future__ import annotations

import json
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer
from typing import Any, Iterator, Optional

from rl_project_b200.serving.api import Router
from rl_project_b200.serving.schemas import error_response

MAX_BODY_BYTES = 8 << 20


def make_handler(router: Router):
    class Handler(BaseHTTPRequestHandler):
        server_version = "forgeline-b200/0.1"
        protocol_version = "HTTP/1.1"

        def _json(self, status: int, payload: Any) -> None:
            data = json.dumps(payload).encode()
            self.send_response(status)
            self.send_header("Content-Type", "application/json")
            self.send_header("Content-Length", str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def _sse(self, lines: Iterator[str]) -> None:
            self.send_response(200)
            self.send_header("Content-Type", "text/event-stream")
            self.send_header("Cache-Control", "no-cache")
            self.send_header("Connection", "close")
            self.end_headers()
            try:
                for line in lines:
                    self.wfile.write(line.encode())
                    self.wfile.flush()
            except Exception as exc:  # noqa: BLE001 - client gone or backend failed mid-stream
                try:
                    self.wfile.write(f"data: {json.dumps(error_response(str(exc), 'server_error', 500))}\n\n".encode())
                except OSError:
                    pass
            self.close_connection = True

        def _dispatch(self, method: str) -> None:
            body = None
            if method == "POST":
                length = int(self.headers.get("Content-Length", 0) or 0)
                if length > MAX_BODY_BYTES:
                    self._json(413, error_response("request body too large", "invalid_request_error", 413))
                    return
                raw = self.rfile.read(length) if length else b""
                try:
                    body = json.loads(raw) if raw else {}
                except json.JSONDecodeError:
                    self._json(400, error_response("invalid JSON body"))
                    return
            status, payload = router.handle(method, self.path.split("?")[0], body)
            if isinstance(payload, dict):
                self._json(status, payload)
            else:
                self._sse(payload)

        def do_GET(self) -> None:  # noqa: N802
            self._dispatch("GET")

        def do_POST(self) -> None:  # noqa: N802
            self._dispatch("POST")

        def log_message(self, format: str, *args: Any) -> None:  # noqa: A002
            pass

    return Handler


class ServingServer:
    def __init__(self, router: Router, host: str = "127.0.0.1", port: int = 8000):
        self.router = router
        self.httpd = ThreadingHTTPServer((host, port), make_handler(router))
        self.httpd.daemon_threads = True
        self._thread: Optional[threading.Thread] = None

    @property
    def port(self) -> int:
        return int(self.httpd.server_address[1])

    def start(self) -> None:
        self._thread = threading.Thread(target=self.httpd.serve_forever, daemon=True, name="forgeline-http")
        self._thread.start()

    def serve_forever(self) -> None:
        self.httpd.serve_forever()

    def stop(self) -> None:
        self.httpd.shutdown()
        self.httpd.server_close()
        if self._thread is not None:
            self._thread.join(timeout=5.0)
