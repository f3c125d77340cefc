"""Rollout engine: sample completions from a policy into ``Trajectory`` objects
(``src/forgeline/rollouts/engine.py`` contract).

Differences by design: ``rollout_many`` generates every prompt x G sample in
one pass (the reference loops prompts one at a time), and ``old_logprobs`` are
recorded here once so algorithms need not run a second old-policy pass.

Generation backend (``RolloutConfig.engine``): ``"auto"`` uses the paged-KV
continuous-batching ``InferenceEngine`` when the policy's model supports it on
a GPU -- all sequences of a rollout decode together whatever their length, and
the G samples of a prompt share one prefill and its KV blocks -- and falls back
to ``policy.generate`` otherwise; ``"generate"`` forces the fallback.  The
inference engine runs the live policy weights, so nothing has to be synced.
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
    engine: str = "auto"  # "auto" | "paged" | "generate"
    engine_max_batch: int = 256  # sequences decoding at once in the paged engine
    engine_kv_blocks: Optional[int] = None  # KV pool size in 16-token blocks (default: enough for max_batch)
    engine_decode_graphs: Optional[bool] = None  # replay decode steps from CUDA graphs (None: RLB_DECODE_GRAPHS, default on)
    # > 0 in a distributed run: the ranks form world / replica_tp tensor-parallel generation replicas of this
    # many GPUs (rollouts/replicas.py) that share each step's prompts; 0: every rank generates its own
    replica_tp: int = 0


class RolloutEngine:
    def __init__(self, policy: PolicyModel, config: RolloutConfig):
        self.policy = policy
        self.cfg = config
        self._engine: Any = None

    # ------------------------------------------------------------ paged inference backend
    def _paged_model(self) -> Any:
        if self.cfg.engine == "generate":
            return None
        model = getattr(self.policy, "model", None)
        ok = model is not None and hasattr(model, "supports_paged_decode") and model.supports_paged_decode()
        if self.cfg.engine == "paged":
            if not ok:
                raise RolloutError("engine='paged' needs a grouped-query TransformerLM policy")
            return model
        return model if ok and next(model.parameters()).is_cuda else None

    def inference_engine(self) -> Any:
        """The paged inference engine over the policy's model (built on first use), or None."""
        if self._engine is None:
            model = self._paged_model()
            if model is None:
                return None
            from rl_project_b200.inference.engine import InferenceEngine

            per_seq = (model.spec.block_size + 15) // 16 + 1
            self._engine = InferenceEngine(model, max_batch=self.cfg.engine_max_batch,
                                           max_blocks=self.cfg.engine_kv_blocks or self.cfg.engine_max_batch * per_seq,
                                           decode_graphs=self.cfg.engine_decode_graphs)
        return self._engine

    def release_engine(self) -> None:
        """Free the paged engine's KV pool (it is rebuilt on the next rollout)."""
        self._engine = None

    def _generate_paged(self, engine: Any, prompts: List[List[int]], G: int,
                        temperature: Optional[float]) -> List[List[int]]:
        from rl_project_b200.inference.requests import SamplingParams

        temp = self.cfg.temperature if temperature is None else temperature
        limit = engine.max_seq_len
        reqs = []
        for p in prompts:
            params = SamplingParams(max_tokens=max(1, min(self.cfg.max_new_tokens, limit - len(p))), temperature=temp,
                                    top_k=self.cfg.top_k, top_p=self.cfg.top_p,
                                    stop_token_ids=[int(t) for t in self.cfg.stop_token_ids])
            reqs.extend(engine.submit(p, params) for _ in range(G))
        was_training = engine.model.training
        try:
            while not all(r.finished for r in reqs):
                engine.step()
        finally:
            engine.model.train(was_training)
        failed = [r for r in reqs if r.error]
        if failed:
            raise RolloutError(f"generation failed: {failed[0].error}")
        return [r.generated_tokens for r in reqs]

    def _old_logprobs(self, prompts: torch.Tensor, responses: torch.Tensor) -> Optional[torch.Tensor]:
        if not self.cfg.record_old_logprobs:
            return None
        return self.policy.logprobs(prompts, responses).detach()

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

    def _to_trajs(self, prompt_ids, responses, old, task, prompt_text, lengths=None) -> List[Trajectory]:
        out = []
        for g in range(responses.shape[0]):
            resp = responses[g, : lengths[g]] if lengths is not None else self._trim(responses[g])
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
        engine = self.inference_engine()
        if engine is not None:
            gen = self._generate_paged(engine, [prompt_ids.tolist()], G, temperature)
            responses = _pad(gen, batch.device, batch.shape[1], SEQ_ALIGN)
            return self._to_trajs(prompt_ids, responses, self._old_logprobs(batch, responses), task, prompt_text,
                                  lengths=[len(g) for g in gen])
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
        engine = self.inference_engine()
        if engine is not None:
            gen = self._generate_paged(engine, [p.tolist() for p in clipped], G, None)
            dev = self.policy.device
            for _, idx in sorted(by_len.items()):
                rows = [gen[i * G + g] for i in idx for g in range(G)]
                responses = _pad(rows, dev, clipped[idx[0]].numel(), SEQ_ALIGN)
                batch = torch.cat([clipped[i].unsqueeze(0).repeat(G, 1) for i in idx], 0).to(dev)
                old = self._old_logprobs(batch, responses)
                for j, i in enumerate(idx):
                    sl = slice(j * G, (j + 1) * G)
                    out[i] = self._to_trajs(clipped[i], responses[sl], old[sl] if old is not None else None,
                                            tasks[i] if tasks else None, prompt_texts[i] if prompt_texts else "",
                                            lengths=[len(r) for r in rows[sl]])
            return out  # type: ignore[return-value]
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


SEQ_ALIGN = 64  # prompt + response batches are right-padded to a multiple of this length


def _aligned_width(prompt_len: int, resp_len: int, align: int) -> int:
    """Response width such that ``prompt_len + width`` is a multiple of ``align``: the attention kernels
    then see few distinct sequence lengths across steps (their per-shape set-up is reused)."""
    if align <= 1:
        return resp_len
    return -(-(prompt_len + resp_len) // align) * align - prompt_len


def _pad(rows: List[List[int]], device: torch.device, prompt_len: int = 0, align: int = 1) -> torch.Tensor:
    R = _aligned_width(prompt_len, max(len(r) for r in rows), align)
    out = torch.zeros((len(rows), R), dtype=torch.long)
    for i, r in enumerate(rows):
        out[i, : len(r)] = torch.as_tensor(r, dtype=torch.long)
    return out.to(device, non_blocking=True)


def stack_group(trajectories: Sequence[Trajectory], pad_value: int = 0, align: int = SEQ_ALIGN):
    """``(prompt [G, P], responses [G, R], mask [G, R])`` for a group sharing one prompt; ``R`` is padded
    so that ``P + R`` is a multiple of ``align`` (the mask marks the real tokens)."""
    prompt = trajectories[0].prompt_ids.unsqueeze(0)
    R = _aligned_width(prompt.shape[1], max(t.response_length for t in trajectories), align)
    G = len(trajectories)
    resp = torch.full((G, R), pad_value, dtype=torch.long)
    mask = torch.zeros((G, R), dtype=torch.float32)
    for i, t in enumerate(trajectories):
        resp[i, : t.response_length] = t.response_ids
        mask[i, : t.response_length] = 1.0
    return prompt.repeat(G, 1), resp, mask


def stack_old_logprobs(trajectories: Sequence[Trajectory], width: Optional[int] = None) -> torch.Tensor:
    R = width if width is not None else max(t.response_length for t in trajectories)
    out = torch.zeros((len(trajectories), R), dtype=torch.float32)
    for i, t in enumerate(trajectories):
        if t.old_logprobs is not None:
            out[i, : t.old_logprobs.numel()] = t.old_logprobs.float()
    return out
