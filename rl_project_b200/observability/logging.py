"""Key/value structured logging.

``get_logger("x").info("event", k=v)`` writes one line, either ``event k=v``
text or a JSON object when ``FORGELINE_LOG_FORMAT=json``; the level comes from
``FORGELINE_LOG_LEVEL`` (same variables as ``src/forgeline/observability/logging.py``).
"""

from __future__ import annotations

import json
import logging
import os
import sys
import time
from typing import Any

ROOT = "forgeline"
_ready = False


def _plain(value: Any) -> Any:
    if value is None or isinstance(value, (str, int, float, bool)):
        return value
    if isinstance(value, (list, tuple)):
        return [_plain(v) for v in value]
    if isinstance(value, dict):
        return {str(k): _plain(v) for k, v in value.items()}
    if hasattr(value, "numel") and hasattr(value, "tolist"):
        return value.item() if value.numel() == 1 else value.tolist()
    return str(value)


class StructuredLogger:
    def __init__(self, name: str):
        self._log = logging.getLogger(name)
        self.name = name

    def _emit(self, level: int, event: str, **kw: Any) -> None:
        if not self._log.isEnabledFor(level):
            return
        if os.environ.get("FORGELINE_LOG_FORMAT", "text") == "json":
            body = {"ts": round(time.time(), 3), "logger": self.name, "event": event}
            body.update({k: _plain(v) for k, v in kw.items()})
            line = json.dumps(body)
        else:
            line = " ".join([event] + [f"{k}={_plain(v)}" for k, v in kw.items()])
        self._log.log(level, line)

    def debug(self, event: str, **kw: Any) -> None:
        self._emit(logging.DEBUG, event, **kw)

    def info(self, event: str, **kw: Any) -> None:
        self._emit(logging.INFO, event, **kw)

    def warning(self, event: str, **kw: Any) -> None:
        self._emit(logging.WARNING, event, **kw)

    def error(self, event: str, **kw: Any) -> None:
        self._emit(logging.ERROR, event, **kw)

    def setLevel(self, level: int) -> None:  # noqa: N802 (logging API name)
        self._log.setLevel(level)


def configure_logging(level: str | int | None = None, stream=None) -> None:
    global _ready
    root = logging.getLogger(ROOT)
    lvl = level if level is not None else os.environ.get("FORGELINE_LOG_LEVEL", "INFO")
    if isinstance(lvl, str):
        lvl = getattr(logging, lvl.upper(), logging.INFO)
    root.setLevel(lvl)
    if not _ready:
        h = logging.StreamHandler(stream or sys.stderr)
        h.setFormatter(logging.Formatter("%(asctime)s %(levelname)s %(name)s: %(message)s", "%H:%M:%S"))
        root.addHandler(h)
        root.propagate = False
        _ready = True


def get_logger(name: str = ROOT) -> StructuredLogger:
    configure_logging()
    full = name if name == ROOT or name.startswith(ROOT + ".") else f"{ROOT}.{name}"
    return StructuredLogger(full)
