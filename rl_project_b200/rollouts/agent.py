"""Multi-turn tool-using rollouts (``src/forgeline/rollouts/agent.py`` behaviour).

The policy writes until it emits ``<tool_call>``; the tool's output is
appended as a ``<tool_result>`` observation (context only, never trained on)
and generation continues until ``<final_answer>`` or the turn budget.  A
trajectory's log-prob is the mean over model segments of each segment's mean
token log-prob, every segment conditioned on the full context before it.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Tuple

import torch

from rl_project_b200.core.errors import ToolExecutionError
from rl_project_b200.core.protocols import GenerationSettings, Trajectory
from rl_project_b200.rollouts.tools.parser import format_tool_result, parse_tagged_output
from rl_project_b200.rollouts.tools.python_executor import PythonExecutorTool

AGENT_SYSTEM_PROMPT = (
    "You solve problems step by step and may run Python.\n"
    "Reason inside <think>...</think>.\n"
    "To run code write <tool_call>{\"name\": \"python_executor\", \"args\": {\"code\": \"...\"}}</tool_call>; "
    "its stdout comes back inside <tool_result>...</tool_result>.\n"
    "Give the answer as <final_answer>...</final_answer>."
)


def build_agent_prompt(problem: str, system_prompt: str = AGENT_SYSTEM_PROMPT) -> str:
    return f"{system_prompt}\n\nProblem: {problem}\n\nSolve step by step:"


@dataclass
class AgentRolloutConfig:
    max_turns: int = 3
    max_new_tokens: int = 128
    temperature: float = 0.9
    max_context_tokens: int = 256
    tools: Dict[str, Callable[[dict], str]] = field(default_factory=lambda: {"python_executor": PythonExecutorTool()})


class AgentRolloutEngine:
    def __init__(self, policy, config: AgentRolloutConfig):
        self.policy = policy
        self.cfg = config

    def _generate_text(self, context: str, temperature: float) -> str:
        ids = torch.tensor(self.policy.encode(context)[-self.cfg.max_context_tokens:], dtype=torch.long)[None]
        with torch.no_grad():
            resp = self.policy.generate(ids.to(self.policy.device),
                                        GenerationSettings(max_new_tokens=self.cfg.max_new_tokens,
                                                           temperature=temperature))
        return self.policy.decode(resp[0])

    def run_episode(self, prompt: str, temperature: Optional[float] = None) -> Tuple[List[str], List[str], str]:
        temp = self.cfg.temperature if temperature is None else temperature
        context, segments, blocks = prompt, [], []
        for _ in range(self.cfg.max_turns + 1):
            seg = self._generate_text(context, temp)
            segments.append(seg)
            parsed = parse_tagged_output(seg)
            if parsed.final_answer is not None:
                context += seg
                break
            call = parsed.tool_call
            if call is None or call.name not in self.cfg.tools:
                context += seg
                break
            try:
                result = self.cfg.tools[call.name](call.args)
            except Exception as exc:  # noqa: BLE001 - a crashing tool becomes an observation
                result = f"ERROR: {ToolExecutionError(str(exc)).message}"
            block = format_tool_result(result)
            blocks.append(block)
            context += seg + block
        return segments, blocks, "".join(segments)

    def rollout(self, task: Dict[str, Any], group_size: int, temperature: Optional[float] = None) -> List[Trajectory]:
        prompt = build_agent_prompt(task["prompt"])
        pids = torch.tensor(self.policy.encode(prompt), dtype=torch.long)
        out = []
        for _ in range(group_size):
            segs, blocks, final = self.run_episode(prompt, temperature)
            rids = torch.tensor(self.policy.encode(final) or [self.policy.pad_token_id], dtype=torch.long)
            out.append(Trajectory(prompt_ids=pids, response_ids=rids, prompt_text=prompt, response_text=final,
                                  task=dict(task), segments=segs, tool_results=blocks,
                                  meta={"n_turns": len(segs), "n_tool_calls": len(blocks)}))
        return out

    def _segment_logprob(self, context: str, segment: str) -> torch.Tensor:
        q = self.policy.encode(context)[-self.cfg.max_context_tokens:]
        r = self.policy.encode(segment)[: self.cfg.max_context_tokens]
        if not q or not r:
            return torch.zeros((), device=self.policy.device)
        block = getattr(getattr(self.policy, "spec", None), "block_size", None)
        if block is not None and len(q) + len(r) > block:
            q = q[-(block - len(r)):] if block > len(r) else q[-1:]
            r = r[: block - len(q)]
        return self.policy.logprobs(torch.tensor(q)[None], torch.tensor(r)[None]).mean()

    def trajectory_logprob(self, trajectory: Trajectory) -> torch.Tensor:
        total = torch.zeros((), device=self.policy.device)
        ctx = trajectory.prompt_text
        for i, seg in enumerate(trajectory.segments):
            total = total + self._segment_logprob(ctx, seg)
            ctx += seg
            if i < len(trajectory.tool_results):
                ctx += trajectory.tool_results[i]
        return total / max(len(trajectory.segments), 1)
