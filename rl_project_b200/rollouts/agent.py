"""Multi-turn tool-using rollouts, advanced in lock-step batches.

Behaviour (the contract of ``src/forgeline/rollouts/agent.py:1-130``): the policy writes until it
emits a ``<tool_call>``; the tool's output joins the context as a ``<tool_result>`` observation
(context only, never trained on) and writing resumes, until ``<final_answer>``, a segment with
neither tag, or ``max_turns`` tool turns.

Design:

* An episode is a small record (context text, segments, observations, live flag).  ``run_episodes``
  advances every live episode of a call by one turn per iteration: ONE batched generation over all
  their contexts (contexts of equal token length share a ``policy.generate`` batch, so the G samples of
  a prompt decode together), then every tool call of that turn runs on a thread pool (the Python
  executor is a subprocess, so calls overlap).  ``run_episode`` is the one-episode case.
* A trajectory's log-prob is the mean over its model segments of each segment's mean token log-prob,
  every segment conditioned on everything before it.  That is ONE forward over the transcript
  (prompt, segments and observations, each encoded on its own and concatenated) because a causal LM
  already conditions each position on its full prefix; ``trajectories_logprob`` batches the
  transcripts of many trajectories into one padded forward.  A transcript longer than the model's
  block keeps its last ``block_size`` tokens; segment tokens cut off are left out of the means.
"""

from __future__ import annotations

from collections import defaultdict
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

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
    tool_workers: int = 8  # threads running one turn's tool calls


@dataclass
class _Episode:
    prompt: str
    segments: List[str] = field(default_factory=list)
    observations: List[str] = field(default_factory=list)
    live: bool = True

    @property
    def context(self) -> str:
        parts = [self.prompt]
        for i, seg in enumerate(self.segments):
            parts.append(seg)
            if i < len(self.observations):
                parts.append(self.observations[i])
        return "".join(parts)

    @property
    def transcript(self) -> str:
        return "".join(self.segments)


def _run_tool(tools: Dict[str, Callable[[dict], str]], name: str, args: dict) -> str:
    try:
        return tools[name](args)
    except Exception as exc:  # noqa: BLE001 - a crashing tool becomes an observation
        return f"ERROR: {ToolExecutionError(str(exc)).message}"


class AgentRolloutEngine:
    def __init__(self, policy, config: AgentRolloutConfig):
        self.policy = policy
        self.cfg = config

    # ------------------------------------------------------------ generation
    def _generate_batch(self, contexts: Sequence[str], temperature: float) -> List[str]:
        """One new segment per context; contexts of equal token length share one generate call."""
        ids = [self.policy.encode(c)[-self.cfg.max_context_tokens:] for c in contexts]
        settings = GenerationSettings(max_new_tokens=self.cfg.max_new_tokens, temperature=temperature)
        by_len: Dict[int, List[int]] = defaultdict(list)
        for i, row in enumerate(ids):
            by_len[len(row)].append(i)
        out: List[str] = [""] * len(contexts)
        dev = self.policy.device
        with torch.no_grad():
            for _, members in sorted(by_len.items()):
                batch = torch.tensor([ids[i] for i in members], dtype=torch.long, device=dev)
                resp = self.policy.generate(batch, settings)
                for row, i in enumerate(members):
                    out[i] = self.policy.decode(resp[row])
        return out

    def run_episodes(self, prompts: Sequence[str], temperature: Optional[float] = None) -> List[Tuple[List[str], List[str], str]]:
        """Run one episode per prompt, all advancing turn by turn together -> ``(segments, observations,
        transcript)`` per prompt, in order."""
        temp = self.cfg.temperature if temperature is None else temperature
        eps = [_Episode(p) for p in prompts]
        for turn in range(self.cfg.max_turns + 1):
            live = [e for e in eps if e.live]
            if not live:
                break
            for e, seg in zip(live, self._generate_batch([e.context for e in live], temp)):
                e.segments.append(seg)
            calls = []
            for e in live:
                parsed = parse_tagged_output(e.segments[-1])
                call = parsed.tool_call
                if parsed.final_answer is not None or call is None or call.name not in self.cfg.tools \
                        or turn == self.cfg.max_turns:
                    e.live = False
                else:
                    calls.append((e, call))
            if calls:
                with ThreadPoolExecutor(max_workers=max(1, min(self.cfg.tool_workers, len(calls)))) as pool:
                    results = list(pool.map(lambda ec: _run_tool(self.cfg.tools, ec[1].name, ec[1].args), calls))
                for (e, _), res in zip(calls, results):
                    e.observations.append(format_tool_result(res))
        return [(e.segments, e.observations, e.transcript) for e in eps]

    def run_episode(self, prompt: str, temperature: Optional[float] = None) -> Tuple[List[str], List[str], str]:
        return self.run_episodes([prompt], temperature)[0]

    def rollout(self, task: Dict[str, Any], group_size: int, temperature: Optional[float] = None) -> List[Trajectory]:
        """``group_size`` episodes of one task, generated as one batch."""
        return self.rollout_many([task], group_size, temperature)[0]

    def rollout_many(self, tasks: Sequence[Dict[str, Any]], group_size: int,
                     temperature: Optional[float] = None) -> List[List[Trajectory]]:
        """``group_size`` episodes for every task, all in one lock-step batch -> one group per task."""
        prompts = [build_agent_prompt(t["prompt"]) for t in tasks]
        results = self.run_episodes([p for p in prompts for _ in range(group_size)], temperature)
        pad = getattr(self.policy, "pad_token_id", 0)
        groups = []
        for ti, (task, prompt) in enumerate(zip(tasks, prompts)):
            pids = torch.tensor(self.policy.encode(prompt), dtype=torch.long)
            grp = []
            for segs, obs, final in results[ti * group_size:(ti + 1) * group_size]:
                rids = torch.tensor(self.policy.encode(final) or [pad], dtype=torch.long)
                grp.append(Trajectory(prompt_ids=pids, response_ids=rids, prompt_text=prompt, response_text=final,
                                      task=dict(task), segments=segs, tool_results=obs,
                                      meta={"n_turns": len(segs), "n_tool_calls": len(obs)}))
            groups.append(grp)
        return groups

    # ------------------------------------------------------------ log-probs
    def _transcript_ids(self, traj: Trajectory) -> Tuple[List[int], List[int]]:
        """Token ids of prompt, segments and observations (each encoded on its own), and per position the index of
        the segment it belongs to (-1: prompt or observation)."""
        ids = list(self.policy.encode(traj.prompt_text))
        owner = [-1] * len(ids)
        for i, seg in enumerate(traj.segments):
            s = self.policy.encode(seg)
            ids += s
            owner += [i] * len(s)
            if i < len(traj.tool_results):
                o = self.policy.encode(traj.tool_results[i])
                ids += o
                owner += [-1] * len(o)
        block = getattr(getattr(self.policy, "spec", None), "block_size", None)
        if block is not None and len(ids) > block:
            ids, owner = ids[-block:], owner[-block:]
        return ids, owner

    def trajectories_logprob(self, trajectories: Sequence[Trajectory]) -> torch.Tensor:
        """``[N]`` trajectory log-probs (see the module docstring) from one padded forward over all transcripts."""
        dev = self.policy.device
        rows = [self._transcript_ids(t) for t in trajectories]
        T = max(max(len(ids) for ids, _ in rows), 2)
        pad = getattr(self.policy, "pad_token_id", 0)
        inp = torch.full((len(rows), T), pad, dtype=torch.long)
        tgt = torch.zeros((len(rows), T), dtype=torch.long)
        own = torch.full((len(rows), T), -1, dtype=torch.long)  # segment of the TARGET token at each position
        for r, (ids, owner) in enumerate(rows):
            n = len(ids)
            inp[r, :n] = torch.tensor(ids)
            if n > 1:
                tgt[r, : n - 1] = torch.tensor(ids[1:])
                own[r, : n - 1] = torch.tensor(owner[1:])
        inp, tgt, own = inp.to(dev), tgt.to(dev), own.to(dev)
        lp = self.policy.token_logprobs(inp, tgt).float()  # [N, T]
        n_seg = max(max((len(t.segments) for t in trajectories), default=1), 1)
        mask = own >= 0
        seg_idx = own.clamp_min(0) + torch.arange(len(rows), device=dev)[:, None] * n_seg
        sums = torch.zeros(len(rows) * n_seg, device=dev).index_add_(0, seg_idx[mask], lp[mask])
        counts = torch.zeros(len(rows) * n_seg, device=dev).index_add_(0, seg_idx[mask], torch.ones_like(lp[mask]))
        sums, counts = sums.view(len(rows), n_seg), counts.view(len(rows), n_seg)
        present = counts > 0
        seg_means = torch.where(present, sums / counts.clamp_min(1), torch.zeros_like(sums))
        return seg_means.sum(1) / present.sum(1).clamp_min(1)

    def trajectory_logprob(self, trajectory: Trajectory) -> torch.Tensor:
        return self.trajectories_logprob([trajectory])[0]
