"""Requests of the inference engine: sampling parameters, a request's life cycle and its token stream.

The public fields (``SamplingParams`` knobs and their validation, ``GenerationRequest.prompt_tokens``,
``params``, ``id``, ``status``, ``generated_tokens``, ``finish_reason``, ``error``, timestamps, ``meta``)
are the interface serving code addresses (reference: ``src/forgeline/inference/requests.py:15-80``).

Life cycle, enforced by a transition table: PENDING -> RUNNING when the scheduler admits the request,
then exactly one terminal state (FINISHED, FAILED, CANCELLED); a waiting request may also go straight to a
terminal state (rejected or cancelled before admission).  Tokens are streamed without a per-token queue:
the engine appends to ``generated_tokens`` under a condition variable and readers keep a cursor into that
list (``read_tokens``), so a reader that falls behind receives the backlog in one batch.
"""

from __future__ import annotations

import threading
import time
import uuid
from dataclasses import dataclass, field
from enum import Enum
from typing import Iterator, List, Optional, Tuple

from rl_project_b200.core.errors import ServingError


class RequestStatus(str, Enum):
    PENDING = "pending"
    RUNNING = "running"
    FINISHED = "finished"
    FAILED = "failed"
    CANCELLED = "cancelled"


_TERMINAL = frozenset({RequestStatus.FINISHED, RequestStatus.FAILED, RequestStatus.CANCELLED})
_ALLOWED = {
    RequestStatus.PENDING: frozenset({RequestStatus.RUNNING}) | _TERMINAL,
    RequestStatus.RUNNING: _TERMINAL,
}


def _in_range(value, lo, hi, lo_open=False) -> bool:
    return (lo < value if lo_open else lo <= value) and value <= hi


@dataclass
class SamplingParams:
    max_tokens: int = 64
    temperature: float = 0.8
    top_k: Optional[int] = 50
    top_p: Optional[float] = None
    min_p: Optional[float] = None
    repetition_penalty: float = 1.0
    stop_token_ids: List[int] = field(default_factory=list)

    def validate(self) -> None:
        problems = []
        if self.max_tokens < 1:
            problems.append("max_tokens must be >= 1")
        if self.temperature < 0:
            problems.append("temperature must be >= 0")
        if self.top_k is not None and self.top_k < 0:
            problems.append("top_k must be >= 0")
        if self.top_p is not None and not _in_range(self.top_p, 0.0, 1.0, lo_open=True):
            problems.append("top_p must be in (0, 1]")
        if self.min_p is not None and not _in_range(self.min_p, 0.0, 1.0):
            problems.append("min_p must be in [0, 1]")
        if self.repetition_penalty <= 0:
            problems.append("repetition_penalty must be > 0")
        if problems:
            raise ServingError("; ".join(problems))

    def filter_key(self) -> tuple:
        """Rows whose keys are equal can be filtered and sampled as one batch."""
        return (self.temperature, self.top_k, self.top_p, self.min_p)


def _new_id() -> str:
    return uuid.uuid4().hex


@dataclass(eq=False)
class GenerationRequest:
    prompt_tokens: List[int]
    params: SamplingParams = field(default_factory=SamplingParams)
    id: str = field(default_factory=_new_id)
    prompt: str = ""
    stream: bool = False
    created_at: float = field(default_factory=time.time)
    status: RequestStatus = RequestStatus.PENDING
    generated_tokens: List[int] = field(default_factory=list)
    finish_reason: Optional[str] = None
    error: Optional[str] = None
    started_at: Optional[float] = None
    finished_at: Optional[float] = None
    meta: dict = field(default_factory=dict)
    _cv: threading.Condition = field(default_factory=threading.Condition, repr=False, compare=False)

    # ------------------------------------------------------------ state
    @property
    def finished(self) -> bool:
        return self.status in _TERMINAL

    @property
    def latency_s(self) -> Optional[float]:
        return None if self.finished_at is None else self.finished_at - self.created_at

    def _move(self, to: RequestStatus) -> None:
        if to not in _ALLOWED.get(self.status, frozenset()):
            raise ServingError(f"request {self.id}: cannot go from {self.status.value} to {to.value}")
        self.status = to

    def start(self) -> None:
        """PENDING -> RUNNING (the scheduler admitted the request)."""
        with self._cv:
            self._move(RequestStatus.RUNNING)
            self.started_at = time.time()

    def push_token(self, token: int) -> None:
        with self._cv:
            self.generated_tokens.append(int(token))
            self._cv.notify_all()

    def finish(self, reason: str, error: Optional[str] = None) -> None:
        """Enter the terminal state ``reason`` implies: FAILED with an error, CANCELLED for "cancelled",
        FINISHED otherwise.  Wakes every reader."""
        to = RequestStatus.FAILED if error else (
            RequestStatus.CANCELLED if reason == "cancelled" else RequestStatus.FINISHED)
        with self._cv:
            self._move(to)
            self.finish_reason, self.error, self.finished_at = reason, error, time.time()
            self._cv.notify_all()

    # ------------------------------------------------------------ streaming
    def read_tokens(self, cursor: int, timeout: Optional[float] = None) -> Tuple[List[int], bool]:
        """Tokens from index ``cursor`` on, waiting (up to ``timeout`` seconds) until there is at least one or
        the request has finished.  Returns ``(tokens, done)``; ``done`` once the request is terminal and every
        token has been handed out."""
        with self._cv:
            if len(self.generated_tokens) <= cursor and not self.finished:
                self._cv.wait_for(lambda: len(self.generated_tokens) > cursor or self.finished, timeout)
            new = self.generated_tokens[cursor:]
            return list(new), self.finished and cursor + len(new) >= len(self.generated_tokens)

    def has_unread(self, cursor: int) -> bool:
        return len(self.generated_tokens) > cursor

    def stream_tokens(self, timeout: Optional[float] = None) -> Iterator[int]:
        """Yield generated tokens as they arrive until the request finishes."""
        cursor, done = 0, False
        while not done:
            new, done = self.read_tokens(cursor, timeout)
            if not new and not done:
                raise TimeoutError(f"request {self.id}: no token within {timeout} s")
            cursor += len(new)
            yield from new
