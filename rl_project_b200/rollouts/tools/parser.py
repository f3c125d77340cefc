"""Tag protocol of agent turns (the tags and dataclasses of ``src/forgeline/rollouts/tools/parser.py``):
``<think>...</think>``, ``<tool_call>{"name": ..., "args": {...}}</tool_call>``, ``<tool_result>`` and
``<final_answer>``.

The text is scanned once with a single pattern that matches any of the four tags (non-greedy body,
closing tag equal to the opening one); the first ``think`` / ``tool_call`` / ``final_answer`` wins and every
``tool_result`` is kept in order.  A tool call counts only if its body is a JSON object with a ``name``.
"""

from __future__ import annotations

import json
import re
from dataclasses import dataclass
from typing import Dict, List, Optional

_ANY_TAG = re.compile(r"<(think|tool_call|tool_result|final_answer)>(.*?)</\1>", re.DOTALL)


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


def _as_call(body: str) -> Optional[ToolCall]:
    try:
        data = json.loads(body)
    except json.JSONDecodeError:
        return None
    if not isinstance(data, dict) or "name" not in data:
        return None
    return ToolCall(str(data["name"]), data.get("args") or {})


def parse_tagged_output(text: str) -> ParsedOutput:
    first: Dict[str, str] = {}
    results: List[str] = []
    for m in _ANY_TAG.finditer(text):
        tag, body = m.group(1), m.group(2).strip()
        if tag == "tool_result":
            results.append(body)
        else:
            first.setdefault(tag, body)
    call = _as_call(first["tool_call"]) if "tool_call" in first else None
    return ParsedOutput(call, first.get("final_answer"), first.get("think"), results, text)


def format_tool_result(text: str) -> str:
    return f"\n<tool_result>\n{text}\n</tool_result>\n"
