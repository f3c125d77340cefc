"""Tag protocol of agent turns: ``<think>``, ``<tool_call>{json}</tool_call>``,
``<tool_result>``, ``<final_answer>`` (``src/forgeline/rollouts/tools/parser.py``)."""

from __future__ import annotations

import json
import re
from dataclasses import dataclass
from typing import List, Optional


def _tag(name: str) -> "re.Pattern[str]":
    return re.compile(rf"<{name}>(.*?)</{name}>", re.DOTALL)


_CALL, _FINAL, _THINK, _RESULT = _tag("tool_call"), _tag("final_answer"), _tag("think"), _tag("tool_result")


@dataclass
class ToolCall:
    name: str
    args: dict


@dataclass
class ParsedOutput:
    tool_call: Optional[ToolCall]
    final_answer: Optional[str]
    thinking: Optional[str]
    tool_results: List[str]
    raw: str


def parse_tagged_output(text: str) -> ParsedOutput:
    call = None
    m = _CALL.search(text)
    if m:
        try:
            data = json.loads(m.group(1).strip())
        except json.JSONDecodeError:
            data = None
        if isinstance(data, dict) and "name" in data:
            call = ToolCall(str(data["name"]), data.get("args", {}) or {})
    fa = _FINAL.search(text)
    th = _THINK.search(text)
    return ParsedOutput(call, fa.group(1).strip() if fa else None, th.group(1).strip() if th else None,
                        [r.group(1).strip() for r in _RESULT.finditer(text)], text)


def format_tool_result(text: str) -> str:
    return f"\n<tool_result>\n{text}\n</tool_result>\n"
