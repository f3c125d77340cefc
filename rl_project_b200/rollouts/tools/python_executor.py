"""Python tool: code runs in a fresh isolated interpreter process with a hard
timeout and a capped output; it never raises (errors become ``ERROR:`` text).
Limits follow ``src/forgeline/rollouts/tools/python_executor.py`` (5 s, 500 chars)."""

from __future__ import annotations

import subprocess
import sys
import textwrap
from dataclasses import dataclass

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
        if self.timed_out:
            return f"ERROR: execution timed out ({TIMEOUT_SEC:.0f}s limit)"
        if self.error and not self.stdout:
            return f"ERROR: {self.stderr[:200]}"
        text = self.stdout[:MAX_OUTPUT_CHARS]
        if self.stderr and not self.error:
            text = text.rstrip() + f"\n# stderr: {self.stderr[:100]}"
        return text


def execute_python(code: str, timeout: float = TIMEOUT_SEC) -> ExecutionResult:
    try:
        r = subprocess.run([sys.executable, "-I", "-c", textwrap.dedent(code)], capture_output=True, text=True,
                           timeout=timeout)
        return ExecutionResult(r.stdout.strip(), r.stderr.strip(), False, r.returncode != 0)
    except subprocess.TimeoutExpired:
        return ExecutionResult("", "", True, True)
    except Exception as exc:  # noqa: BLE001
        return ExecutionResult("", str(exc), False, True)


class PythonExecutorTool:
    name = "python_executor"
    description = "Executes Python code and returns stdout."

    def __init__(self, timeout: float = TIMEOUT_SEC):
        self.timeout = timeout

    def __call__(self, args: dict) -> str:
        code = args.get("code", "print('')") if isinstance(args, dict) else str(args)
        return execute_python(code, timeout=self.timeout).output
