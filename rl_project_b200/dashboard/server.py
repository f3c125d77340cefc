"""Local read-only dashboard server (standard library only).

GET endpoints: ``/`` (single-page UI, no external assets), ``/health``,
``/api/overview``, ``/api/runs``, ``/api/runs/<id>``, ``/api/registry``,
``/api/benchmarks``, ``/api/inspect?checkpoint=<dir>&text=<prompt>`` (only
checkpoints under a configured runs root).  Nothing is ever written; registry
changes go through the ``registry`` CLI command.
"""

from __future__ import annotations

import json
import threading
from collections import OrderedDict
from importlib import resources
from pathlib import Path
from typing import Any, Dict, Optional, Tuple
from urllib.parse import parse_qs, urlparse

from rl_project_b200.dashboard import data
from rl_project_b200.dashboard.data import DashboardSources
from rl_project_b200.serving.http import AsyncHTTPServer

JSON = "application/json"


def index_html() -> str:
    return resources.files("rl_project_b200.dashboard").joinpath("static/index.html").read_text()


class DashboardApp:
    """Routes a GET path to the data layer; ``handle`` is usable without sockets."""

    def __init__(self, sources: DashboardSources, inspect_cache_size: int = 4):
        self.sources = sources
        self._cache: "OrderedDict[Tuple[str, str], Any]" = OrderedDict()
        self._cache_size = inspect_cache_size
        self._lock = threading.Lock()

    def _run_path(self, run_id: str) -> Optional[str]:
        return next((r["path"] for r in data.discover_runs(self.sources.runs) if r["id"] == run_id), None)

    def _inspect(self, query) -> Tuple[int, str, Any]:
        ckpt = (query.get("checkpoint") or [""])[0]
        text = (query.get("text") or [""])[0][:2000]
        if not ckpt or not self.sources.checkpoint_allowed(ckpt):
            return 403, JSON, {"error": "checkpoint must be a checkpoint directory under a configured runs root"}
        key = (str(Path(ckpt).resolve()), text)
        with self._lock:
            hit = self._cache.get(key)
        if hit is None:
            try:
                hit = data.inspect_checkpoint(ckpt, text=text)
            except Exception as exc:  # noqa: BLE001
                return 422, JSON, {"error": f"{type(exc).__name__}: {exc}"}
            with self._lock:
                self._cache[key] = hit
                while len(self._cache) > self._cache_size:
                    self._cache.popitem(last=False)
        return 200, JSON, hit

    def handle(self, path: str) -> Tuple[int, str, Any]:
        url = urlparse(path)
        route, query = url.path.rstrip("/") or "/", parse_qs(url.query)
        s = self.sources
        if route in ("/", "/index.html"):
            return 200, "text/html; charset=utf-8", index_html()
        if route == "/health":
            return 200, JSON, {"status": "ok"}
        if route == "/api/overview":
            benches = data.benchmark_records(s.benchmarks)
            return 200, JSON, {"sources": {"runs": s.runs, "registry": s.registry, "benchmarks": s.benchmarks},
                               "runs": data.discover_runs(s.runs), "registry": data.registry_view(s.registry),
                               "benchmarks": [{k: b[k] for k in ("record", "evidence", "revalidation_recommended",
                                                                 "published")} for b in benches]}
        if route == "/api/runs":
            return 200, JSON, data.discover_runs(s.runs)
        if route.startswith("/api/runs/"):
            run_path = self._run_path(route.rsplit("/", 1)[-1])
            if run_path is None:
                return 404, JSON, {"error": "unknown run"}
            return 200, JSON, data.run_detail(run_path)
        if route == "/api/registry":
            return 200, JSON, data.registry_view(s.registry)
        if route == "/api/benchmarks":
            return 200, JSON, data.benchmark_records(s.benchmarks)
        if route == "/api/inspect":
            return self._inspect(query)
        return 404, JSON, {"error": f"no route {route}"}


class DashboardServer:
    """The dashboard's read-only views over the shared asyncio HTTP core (GET only; file-system reads run in
    its thread pool)."""

    def __init__(self, app: DashboardApp, host: str = "127.0.0.1", port: int = 8765):
        self.app = app
        self._http = AsyncHTTPServer(self._serve, host, port, workers=4, server_name="forgeline-b200-dashboard/0.1",
                                     on_bad_request=lambda status, msg: json.dumps({"error": msg}).encode(),
                                     extra_headers={"Cache-Control": "no-store"})
        self.host, self.port = host, self._http.port

    def _serve(self, method: str, target: str, headers: Dict[str, str], body: bytes):
        if method != "GET":
            return 404, "application/json", json.dumps({"error": f"no route for {method}"}).encode()
        status, ctype, payload = self.app.handle(target)
        data = payload.encode() if isinstance(payload, str) else json.dumps(payload, default=str).encode()
        return status, ctype, data

    @property
    def url(self) -> str:
        return f"http://{self.host}:{self.port}"

    def start(self) -> "DashboardServer":
        self._http.start("forgeline-dashboard")
        return self

    def serve_forever(self) -> None:
        self._http.serve_forever()

    def stop(self) -> None:
        self._http.stop()
