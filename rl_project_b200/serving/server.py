"""HTTP/1.1 front end of the router on one asyncio event loop.

Design: a single event loop (its own thread, or the caller's with ``serve_forever``) owns every connection;
the router and its backends -- which block on the GPU engine -- run in a small thread pool, so a slow
generation never holds up the loop.  A streamed completion is pulled from the backend's iterator one piece
at a time in that pool and each Server-Sent-Events line is written and drained as it arrives, so the
client sees tokens at the engine's pace.  JSON responses keep the connection open (HTTP/1.1 keep-alive); an
event stream ends it.  The routes, status codes and wire format are the router's (``serving/api.py``).
"""

from __future__ import annotations

import asyncio
import json
import threading
from concurrent.futures import ThreadPoolExecutor
from typing import Any, Dict, Iterator, Optional, Tuple

from rl_project_b200.serving.api import Router
from rl_project_b200.serving.schemas import error_response

MAX_BODY_BYTES = 8 << 20
MAX_HEADER_BYTES = 64 << 10
_REASONS = {200: "OK", 400: "Bad Request", 404: "Not Found", 413: "Payload Too Large", 500: "Internal Server Error",
            503: "Service Unavailable"}
_DONE = object()


class _BadRequest(Exception):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


async def _read_request(reader: asyncio.StreamReader) -> Optional[Tuple[str, str, Dict[str, str], bytes]]:
    """One request: (method, path without query, lower-cased headers, body); None at end of stream."""
    try:
        head = await reader.readuntil(b"\r\n\r\n")
    except asyncio.IncompleteReadError:
        return None
    except asyncio.LimitOverrunError:
        raise _BadRequest(400, "request head too large")
    lines = head.decode("latin-1").split("\r\n")
    parts = lines[0].split(" ")
    if len(parts) != 3:
        raise _BadRequest(400, "malformed request line")
    headers = {}
    for ln in lines[1:]:
        if ":" in ln:
            k, v = ln.split(":", 1)
            headers[k.strip().lower()] = v.strip()
    length = int(headers.get("content-length", "0") or 0)
    if length > MAX_BODY_BYTES:
        raise _BadRequest(413, "request body too large")
    body = await reader.readexactly(length) if length else b""
    return parts[0].upper(), parts[1].split("?")[0], headers, body


def _head(status: int, headers: Dict[str, str]) -> bytes:
    lines = [f"HTTP/1.1 {status} {_REASONS.get(status, 'Status')}", "Server: forgeline-b200/0.1"]
    lines += [f"{k}: {v}" for k, v in headers.items()]
    return ("\r\n".join(lines) + "\r\n\r\n").encode("latin-1")


class ServingServer:
    """``start()`` serves on a background thread, ``serve_forever()`` on the caller's; ``port`` is the bound
    port (``port=0`` picks a free one); ``stop()`` closes the listener and the loop."""

    def __init__(self, router: Router, host: str = "127.0.0.1", port: int = 8000, workers: int = 8):
        self.router = router
        self.host, self._want_port = host, port
        self._pool = ThreadPoolExecutor(max_workers=workers, thread_name_prefix="forgeline-serve")
        self._loop = asyncio.new_event_loop()
        self._server: Optional[asyncio.base_events.Server] = None
        self._thread: Optional[threading.Thread] = None
        # bind now, so the port is known before the loop runs (and a busy port fails here)
        self._server = self._loop.run_until_complete(
            asyncio.start_server(self._connection, host, port, limit=MAX_HEADER_BYTES))

    @property
    def port(self) -> int:
        return int(self._server.sockets[0].getsockname()[1])

    def start(self) -> None:
        self._thread = threading.Thread(target=self._run, daemon=True, name="forgeline-http")
        self._thread.start()

    def serve_forever(self) -> None:
        self._run()

    def _run(self) -> None:
        asyncio.set_event_loop(self._loop)
        self._loop.run_forever()

    def stop(self) -> None:
        async def close():
            self._server.close()
            await self._server.wait_closed()

        if self._loop.is_running():
            asyncio.run_coroutine_threadsafe(close(), self._loop).result(timeout=5.0)
            self._loop.call_soon_threadsafe(self._loop.stop)
        else:
            self._loop.run_until_complete(close())
        if self._thread is not None:
            self._thread.join(timeout=5.0)
        self._pool.shutdown(wait=False, cancel_futures=True)
        if not self._loop.is_running():
            self._loop.close()

    # ------------------------------------------------------------------ connections
    async def _connection(self, reader: asyncio.StreamReader, writer: asyncio.StreamWriter) -> None:
        loop = asyncio.get_running_loop()
        try:
            while True:
                try:
                    req = await _read_request(reader)
                except _BadRequest as exc:
                    await self._json(writer, exc.status, error_response(str(exc), "invalid_request_error", exc.status),
                                     keep=False)
                    return
                if req is None:
                    return
                method, path, headers, raw = req
                body = None
                if method == "POST":
                    try:
                        body = json.loads(raw) if raw else {}
                    except json.JSONDecodeError:
                        await self._json(writer, 400, error_response("invalid JSON body"), keep=False)
                        return
                status, payload = await loop.run_in_executor(self._pool, self.router.handle, method, path, body)
                if isinstance(payload, dict):
                    keep = headers.get("connection", "keep-alive").lower() != "close"
                    await self._json(writer, status, payload, keep)
                    if not keep:
                        return
                else:
                    await self._stream(writer, payload)
                    return
        except (ConnectionError, asyncio.IncompleteReadError):
            pass
        finally:
            writer.close()

    async def _json(self, writer: asyncio.StreamWriter, status: int, payload: Any, keep: bool) -> None:
        data = json.dumps(payload).encode()
        writer.write(_head(status, {"Content-Type": "application/json", "Content-Length": str(len(data)),
                                    "Connection": "keep-alive" if keep else "close"}) + data)
        await writer.drain()

    async def _stream(self, writer: asyncio.StreamWriter, lines: Iterator[str]) -> None:
        """Server-Sent Events: each line pulled from the backend in the pool, written and drained at once; a
        failure mid-stream becomes a final error event."""
        loop = asyncio.get_running_loop()
        writer.write(_head(200, {"Content-Type": "text/event-stream", "Cache-Control": "no-cache",
                                 "Connection": "close"}))
        await writer.drain()
        it = iter(lines)
        try:
            while True:
                line = await loop.run_in_executor(self._pool, next, it, _DONE)
                if line is _DONE:
                    break
                writer.write(line.encode())
                await writer.drain()
        except ConnectionError:
            return
        except Exception as exc:  # noqa: BLE001 - backend failed mid-stream
            writer.write(f"data: {json.dumps(error_response(str(exc), 'server_error', 500))}\n\n".encode())
            await writer.drain()
