"""Python tool for agent rollouts: each snippet runs in a fresh isolated interpreter (``python -I``) with a
hard timeout and a capped output, and the call never raises -- failures come back as ``ERROR: ...`` text
(limits and messages of ``src/forgeline/rollouts/tools/python_executor.py``: 5 s, 500 characters).

``execute_many`` serves lock-step batched rollouts: it starts every snippet's interpreter at once and
collects them against one shared deadline, so a turn of ``n`` tool calls costs about one timeout, not
``n``.
"""

from __future__ import annotations

import subprocess
import sys
import textwrap
import time
from dataclasses import dataclass
from typing import List, Sequence

TIMEOUT_SEC = 5.0
MAX_OUTPUT_CHARS = 500


@dataclass
class ExecutionResult:
    stdout: str
    stderr: str
    timed_out: bool
    error: bool

    @property
    def output(self) -> str:
        """What the model sees: stdout (capped), a stderr note on success, or an error line."""
        if self.timed_out:
            return f"ERROR: execution timed out ({TIMEOUT_SEC:.0f}s limit)"
        if self.error and not self.stdout:
            return f"ERROR: {self.stderr[:200]}"
        shown = self.stdout[:MAX_OUTPUT_CHARS]
        return shown if not self.stderr or self.error else shown.rstrip() + f"\n# stderr: {self.stderr[:100]}"


def _start(code: str) -> subprocess.Popen:
    return subprocess.Popen([sys.executable, "-I", "-c", textwrap.dedent(code)], stdout=subprocess.PIPE,
                            stderr=subprocess.PIPE, stdin=subprocess.DEVNULL, text=True)


def _finish(proc: subprocess.Popen, remaining: float) -> ExecutionResult:
    try:
        out, err = proc.communicate(timeout=max(remaining, 0.0))
    except subprocess.TimeoutExpired:
        proc.kill()
        proc.communicate()
        return ExecutionResult("", "", True, True)
    return ExecutionResult(out.strip(), err.strip(), False, proc.returncode != 0)


def execute_many(codes: Sequence[str], timeout: float = TIMEOUT_SEC) -> List[ExecutionResult]:
    """Run every snippet concurrently; each gets at most ``timeout`` seconds from the common start."""
    procs: List[object] = []
    for code in codes:
        try:
            procs.append(_start(code))
        except Exception as exc:  # noqa: BLE001 - a snippet that cannot start is an error result
            procs.append(ExecutionResult("", str(exc), False, True))
    deadline = time.monotonic() + timeout
    return [p if isinstance(p, ExecutionResult) else _finish(p, deadline - time.monotonic()) for p in procs]


def execute_python(code: str, timeout: float = TIMEOUT_SEC) -> ExecutionResult:
    return execute_many([code], timeout)[0]


def _code_of(args) -> str:
    return args.get("code", "print('')") if isinstance(args, dict) else str(args)


class PythonExecutorTool:
    name = "python_executor"
    description = "Executes Python code and returns stdout."

    def __init__(self, timeout: float = TIMEOUT_SEC):
        self.timeout = timeout

    def __call__(self, args: dict) -> str:
        return execute_python(_code_of(args), timeout=self.timeout).output

    def call_many(self, arg_list: Sequence[dict]) -> List[str]:
        """One output per call, the interpreters running side by side."""
        return [r.output for r in execute_many([_code_of(a) for a in arg_list], self.timeout)]
