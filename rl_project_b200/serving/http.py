"""Minimal HTTP/1.1 server core on one asyncio event loop, shared by the serving API and the dashboard.

One loop (its own thread after ``start()``, or the caller's with ``serve_forever()``) owns every
connection; the application callable -- which may block on the GPU engine or the file system -- runs in a
thread pool, so one slow request never holds up the others.  The callable gets ``(method, target, headers,
body)`` (target with its query string, lower-cased header names, raw body bytes) and returns ``(status,
content type, payload)``: ``bytes`` are sent with a Content-Length and the connection kept alive (HTTP/1.1),
an iterator of ``str`` is sent as it is produced (each piece pulled in the pool, written and drained at once:
Server-Sent Events) and then the connection is closed.
"""

from __future__ import annotations

import asyncio
import threading
from concurrent.futures import ThreadPoolExecutor
from typing import Callable, Dict, Iterator, Optional, Tuple, Union

MAX_BODY_BYTES = 8 << 20
MAX_HEADER_BYTES = 64 << 10
_REASONS = {200: "OK", 400: "Bad Request", 404: "Not Found", 413: "Payload Too Large", 500: "Internal Server Error",
            503: "Service Unavailable"}
_END = object()

Payload = Union[bytes, Iterator[str]]
App = Callable[[str, str, Dict[str, str], bytes], Tuple[int, str, Payload]]


class HTTPError(Exception):
    """Raised while reading a request: answered with ``status`` and the connection closed."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


async def read_request(reader: asyncio.StreamReader) -> Optional[Tuple[str, str, Dict[str, str], bytes]]:
    """One request: (method, target, lower-cased headers, body); None when the client closed the connection."""
    try:
        head = await reader.readuntil(b"\r\n\r\n")
    except asyncio.IncompleteReadError:
        return None
    except asyncio.LimitOverrunError:
        raise HTTPError(400, "request head too large")
    lines = head.decode("latin-1").split("\r\n")
    parts = lines[0].split(" ")
    if len(parts) != 3:
        raise HTTPError(400, "malformed request line")
    headers = {}
    for ln in lines[1:]:
        if ":" in ln:
            k, v = ln.split(":", 1)
            headers[k.strip().lower()] = v.strip()
    length = int(headers.get("content-length", "0") or 0)
    if length > MAX_BODY_BYTES:
        raise HTTPError(413, "request body too large")
    body = await reader.readexactly(length) if length else b""
    return parts[0].upper(), parts[1], headers, body


def response_head(status: int, headers: Dict[str, str], server: str) -> bytes:
    lines = [f"HTTP/1.1 {status} {_REASONS.get(status, 'Status')}", f"Server: {server}"]
    lines += [f"{k}: {v}" for k, v in headers.items()]
    return ("\r\n".join(lines) + "\r\n\r\n").encode("latin-1")


class AsyncHTTPServer:
    """Binds at construction (``port=0`` picks a free port, a busy port fails here); ``start`` / ``serve_forever``
    run the loop; ``stop`` closes the listener, the loop and the pool."""

    def __init__(self, app: App, host: str = "127.0.0.1", port: int = 8000, workers: int = 8,
                 server_name: str = "forgeline-b200/0.1", on_bad_request: Optional[Callable[[int, str], bytes]] = None,
                 extra_headers: Optional[Dict[str, str]] = None):
        self.app, self.host, self.server_name = app, host, server_name
        self.on_bad_request = on_bad_request or (lambda status, msg: msg.encode())
        self.extra_headers = dict(extra_headers or {})
        self._pool = ThreadPoolExecutor(max_workers=workers, thread_name_prefix="forgeline-http")
        self._loop = asyncio.new_event_loop()
        self._thread: Optional[threading.Thread] = None
        self._server = self._loop.run_until_complete(
            asyncio.start_server(self._connection, host, port, limit=MAX_HEADER_BYTES))

    @property
    def port(self) -> int:
        return int(self._server.sockets[0].getsockname()[1])

    def start(self, name: str = "forgeline-http") -> None:
        self._thread = threading.Thread(target=self._run, daemon=True, name=name)
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

    async def _connection(self, reader: asyncio.StreamReader, writer: asyncio.StreamWriter) -> None:
        loop = asyncio.get_running_loop()
        try:
            while True:
                try:
                    req = await read_request(reader)
                except HTTPError as exc:
                    await self._send(writer, exc.status, "application/json", self.on_bad_request(exc.status, str(exc)),
                                     keep=False)
                    return
                if req is None:
                    return
                method, target, headers, body = req
                status, ctype, payload = await loop.run_in_executor(self._pool, self.app, method, target, headers, body)
                if isinstance(payload, (bytes, bytearray)):
                    keep = headers.get("connection", "keep-alive").lower() != "close"
                    await self._send(writer, status, ctype, bytes(payload), keep)
                    if not keep:
                        return
                else:
                    await self._stream(writer, status, ctype, payload)
                    return
        except (ConnectionError, asyncio.IncompleteReadError):
            pass
        finally:
            writer.close()

    async def _send(self, writer, status: int, ctype: str, data: bytes, keep: bool) -> None:
        headers = {"Content-Type": ctype, "Content-Length": str(len(data)), **self.extra_headers,
                   "Connection": "keep-alive" if keep else "close"}
        writer.write(response_head(status, headers, self.server_name) + data)
        await writer.drain()

    async def _stream(self, writer, status: int, ctype: str, pieces: Iterator[str]) -> None:
        loop = asyncio.get_running_loop()
        writer.write(response_head(status, {"Content-Type": ctype, "Cache-Control": "no-cache", "Connection": "close"},
                                   self.server_name))
        await writer.drain()
        it = iter(pieces)
        try:
            while True:
                piece = await loop.run_in_executor(self._pool, next, it, _END)
                if piece is _END:
                    break
                writer.write(piece.encode())
                await writer.drain()
        except ConnectionError:
            return
        except Exception as exc:  # noqa: BLE001 - the producer failed mid-stream: tell the client, then close
            writer.write(b"data: " + self.on_bad_request(500, str(exc)) + b"\n\n")
            await writer.drain()
