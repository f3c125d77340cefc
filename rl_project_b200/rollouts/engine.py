"""Rollout engine: sample completions from a policy into ``Trajectory`` objects
(``src/forgeline/rollouts/engine.py`` contract).

Differences by design: ``rollout_many`` batches every prompt x G sample into
one generation call per prompt length (the reference loops prompts one at a
time), and ``old_logprobs`` are recorded here once so algorithms need not run a
second old-policy pass.
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Sequence

import torch

from rl_project_b200.core.errors import RolloutError
from rl_project_b200.core.protocols import GenerationSettings, PolicyModel, Trajectory
from rl_project_b200.observability.logging import get_logger

log = get_logger("rollouts")


@dataclass
class RolloutConfig:
    group_size: int = 4
    max_new_tokens: int = 64
    temperature: float = 0.8
    top_k: Optional[int] = None
    top_p: Optional[float] = None
    max_prompt_length: int = 128
    record_old_logprobs: bool = True
    stop_token_ids: Sequence[int] = ()


class RolloutEngine:
    def __init__(self, policy: PolicyModel, config: RolloutConfig):
        self.policy = policy
        self.cfg = config

    def _settings(self, temperature: Optional[float] = None) -> GenerationSettings:
        return GenerationSettings(max_new_tokens=self.cfg.max_new_tokens,
                                  temperature=self.cfg.temperature if temperature is None else temperature,
                                  top_k=self.cfg.top_k, top_p=self.cfg.top_p,
                                  stop_token_ids=tuple(self.cfg.stop_token_ids))

    def _trim(self, resp: torch.Tensor) -> torch.Tensor:
        stop = {int(t) for t in self.cfg.stop_token_ids}
        if stop:
            hits = [i for i, t in enumerate(resp.tolist()) if int(t) in stop]
            if hits:
                return resp[: hits[0] + 1]
        return resp

    @torch.no_grad()
    def _sample(self, prompts: torch.Tensor, temperature: Optional[float] = None):
        try:
            responses = self.policy.generate(prompts, self._settings(temperature))
        except Exception as exc:  # noqa: BLE001
            raise RolloutError(f"generation failed: {type(exc).__name__}: {exc}") from exc
        if responses.shape[1] == 0:
            raise RolloutError("policy produced an empty response",
                               hint="Increase max_new_tokens or check the prompt length vs block_size.")
        old = self.policy.logprobs(prompts, responses).detach() if self.cfg.record_old_logprobs else None
        return responses, old

    def _to_trajs(self, prompt_ids, responses, old, task, prompt_text) -> List[Trajectory]:
        out = []
        for g in range(responses.shape[0]):
            resp = self._trim(responses[g])
            out.append(Trajectory(prompt_ids=prompt_ids.detach().cpu(), response_ids=resp.detach().cpu(),
                                  prompt_text=prompt_text, response_text=self._decode(resp), task=dict(task or {}),
                                  truncated=bool(resp.numel() >= self.cfg.max_new_tokens),
                                  old_logprobs=old[g, : resp.numel()].float().cpu() if old is not None else None))
        return out

    @torch.no_grad()
    def rollout(self, prompt_ids: torch.Tensor, task: Optional[Dict[str, Any]] = None, prompt_text: str = "",
                group_size: Optional[int] = None, temperature: Optional[float] = None) -> List[Trajectory]:
        G = group_size or self.cfg.group_size
        prompt_ids = prompt_ids[-self.cfg.max_prompt_length:]
        if prompt_ids.numel() == 0:
            raise RolloutError("empty prompt")
        batch = prompt_ids.unsqueeze(0).repeat(G, 1).to(self.policy.device)
        responses, old = self._sample(batch, temperature)
        return self._to_trajs(prompt_ids, responses, old, task, prompt_text)

    @torch.no_grad()
    def rollout_many(self, prompts: Sequence[torch.Tensor], tasks: Optional[Sequence[Dict[str, Any]]] = None,
                     prompt_texts: Optional[Sequence[str]] = None,
                     group_size: Optional[int] = None) -> List[List[Trajectory]]:
        """All prompts x G samples; prompts of equal length share one generation batch."""
        G = group_size or self.cfg.group_size
        clipped = [p[-self.cfg.max_prompt_length:] for p in prompts]
        by_len: Dict[int, List[int]] = defaultdict(list)
        for i, p in enumerate(clipped):
            if p.numel() == 0:
                raise RolloutError("empty prompt")
            by_len[p.numel()].append(i)
        out: List[Optional[List[Trajectory]]] = [None] * len(prompts)
        for _, idx in sorted(by_len.items()):
            batch = torch.cat([clipped[i].unsqueeze(0).repeat(G, 1) for i in idx], 0).to(self.policy.device)
            responses, old = self._sample(batch)
            for j, i in enumerate(idx):
                sl = slice(j * G, (j + 1) * G)
                out[i] = self._to_trajs(clipped[i], responses[sl], old[sl] if old is not None else None,
                                        tasks[i] if tasks else None, prompt_texts[i] if prompt_texts else "")
        return out  # type: ignore[return-value]

    def _decode(self, ids: torch.Tensor) -> str:
        dec = getattr(self.policy, "decode", None)
        return dec(ids) if dec is not None else ""


def stack_group(trajectories: Sequence[Trajectory], pad_value: int = 0):
    """``(prompt [G, P], responses [G, R], mask [G, R])`` for a group sharing one prompt."""
    prompt = trajectories[0].prompt_ids.unsqueeze(0)
    R = max(t.response_length for t in trajectories)
    G = len(trajectories)
    resp = torch.full((G, R), pad_value, dtype=torch.long)
    mask = torch.zeros((G, R), dtype=torch.float32)
    for i, t in enumerate(trajectories):
        resp[i, : t.response_length] = t.response_ids
        mask[i, : t.response_length] = 1.0
    return prompt.repeat(G, 1), resp, mask


def stack_old_logprobs(trajectories: Sequence[Trajectory]) -> torch.Tensor:
    R = max(t.response_length for t in trajectories)
    out = torch.zeros((len(trajectories), R), dtype=torch.float32)
    for i, t in enumerate(trajectories):
        if t.old_logprobs is not None:
            out[i, : t.old_logprobs.numel()] = t.old_logprobs.float()
    return out
