"""Serving backends: text in, text out, over the inference engine.

``EngineBackend`` tokenizes, submits to an ``InferenceEngine`` (driven by the
engine's background thread, or inline when ``background=False``), waits on
the request's token queue -- no polling -- and detokenizes; stop strings end a
completion at their first occurrence.  ``EchoBackend`` is the deterministic
test double (prompt reversed, cut to ``max_tokens`` characters), as in
``src/forgeline/serving/backends.py:108-131``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Dict, Iterator, List, Optional, Protocol, Sequence

from rl_project_b200.core.errors import BackendUnavailableError, ServingError
from rl_project_b200.inference.requests import GenerationRequest, SamplingParams


@dataclass
class CompletionResult:
    text: str
    prompt_tokens: int
    completion_tokens: int
    finish_reason: str
    backend: str
    request_id: str


class Backend(Protocol):
    name: str

    def complete(self, prompt: str, params: SamplingParams, request_id: Optional[str] = None,
                 stop: Sequence[str] = ()) -> CompletionResult: ...

    def stream(self, prompt: str, params: SamplingParams, request_id: Optional[str] = None,
               stop: Sequence[str] = ()) -> Iterator[str]: ...

    def healthy(self) -> bool: ...


class _Toggle:
    _enabled = True

    def healthy(self) -> bool:
        return self._enabled

    def disable(self) -> None:
        self._enabled = False

    def enable(self) -> None:
        self._enabled = True

    def _check(self) -> None:
        if not self._enabled:
            raise BackendUnavailableError(f"backend {self.name!r} is disabled")  # type: ignore[attr-defined]


def _cut_at_stop(text: str, stop: Sequence[str]) -> Optional[int]:
    hits = [text.find(s) for s in stop if s and s in text]
    return min(hits) if hits else None


def _stop_prefix_len(text: str, stop: Sequence[str]) -> int:
    """Length of the longest suffix of ``text`` that starts some stop string."""
    best = 0
    for s in stop:
        for k in range(min(len(s) - 1, len(text)), best, -1):
            if text.endswith(s[:k]):
                best = k
                break
    return best


class EngineBackend(_Toggle):
    def __init__(self, name: str, engine: Any, tokenizer: Any, background: bool = True):
        self.name = name
        self.engine = engine
        self.tokenizer = tokenizer
        self._background = background
        self._enabled = True
        if background:
            engine.start()

    def _submit(self, prompt: str, params: SamplingParams, request_id: Optional[str]) -> GenerationRequest:
        self._check()
        ids = self.tokenizer.encode(prompt)
        if not ids:
            raise ServingError("prompt produced no tokens under this tokenizer")
        kwargs: Dict[str, Any] = {"prompt": prompt}
        if request_id:
            kwargs["id"] = request_id
        return self.engine.submit(ids, params, **kwargs)

    def _tokens(self, req: GenerationRequest) -> Iterator[int]:
        """The request's tokens as they are produced: a cursor into its token list, stepping the engine
        from this thread when no background loop drives it."""
        cursor = 0
        while True:
            if not self._background and not req.finished and not req.has_unread(cursor):
                self.engine.step()
                continue
            new, done = req.read_tokens(cursor, timeout=None if self._background else 0)
            cursor += len(new)
            yield from new
            if done:
                return

    def complete(self, prompt: str, params: SamplingParams, request_id: Optional[str] = None,
                 stop: Sequence[str] = ()) -> CompletionResult:
        req = self._submit(prompt, params, request_id)
        tokens: List[int] = []
        finish = None
        for tok in self._tokens(req):
            tokens.append(tok)
            if stop and _cut_at_stop(self.tokenizer.decode(tokens), stop) is not None:
                self.engine.cancel(req.id)
                finish = "stop"
                break
        if req.error:
            raise ServingError(f"generation failed: {req.error}")
        text = self.tokenizer.decode(tokens)
        cut = _cut_at_stop(text, stop) if stop else None
        if cut is not None:
            text, finish = text[:cut], "stop"
        return CompletionResult(text=text, prompt_tokens=len(req.prompt_tokens), completion_tokens=len(tokens),
                                finish_reason=finish or req.finish_reason or "length", backend=self.name,
                                request_id=req.id)

    def stream(self, prompt: str, params: SamplingParams, request_id: Optional[str] = None,
               stop: Sequence[str] = ()) -> Iterator[str]:
        req = self._submit(prompt, params, request_id)
        pending: List[int] = []
        buf = ""  # decoded text not yet yielded (may hold the start of a stop string)
        for tok in self._tokens(req):
            pending.append(tok)
            text = self.tokenizer.decode(pending)
            if not text or "\ufffd" in text:  # wait until the bytes decode to whole characters
                continue
            pending = []
            buf += text
            if stop:
                cut = _cut_at_stop(buf, stop)
                if cut is not None:
                    if cut:
                        yield buf[:cut]
                    self.engine.cancel(req.id)
                    return
                hold = _stop_prefix_len(buf, stop)
                out, buf = buf[: len(buf) - hold], buf[len(buf) - hold:]
                if out:
                    yield out
            else:
                yield buf
                buf = ""
        if buf:
            yield buf
        if req.error:
            raise ServingError(f"generation failed: {req.error}")

    def close(self) -> None:
        self.engine.stop()


class EchoBackend(_Toggle):
    name = "echo"

    def __init__(self, name: str = "echo"):
        self.name = name
        self._enabled = True

    def complete(self, prompt: str, params: SamplingParams, request_id: Optional[str] = None,
                 stop: Sequence[str] = ()) -> CompletionResult:
        self._check()
        text = prompt[::-1][: params.max_tokens]
        return CompletionResult(text=text, prompt_tokens=len(prompt), completion_tokens=len(text),
                                finish_reason="length", backend=self.name, request_id=request_id or "echo")

    def stream(self, prompt: str, params: SamplingParams, request_id: Optional[str] = None,
               stop: Sequence[str] = ()) -> Iterator[str]:
        yield from self.complete(prompt, params, request_id).text
