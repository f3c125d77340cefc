"""Group Relative Policy Optimization (single-turn and tool-using agent mode).

Semantics of ``src/forgeline/training/grpo.py``: G samples per prompt,
advantages ``(r - mean) / (std + eps)`` within the group, ``objective``
``clipped`` (PPO surrogate + ``kl_coef * clamp(mean(ref - new), 0)`` with the
clamp applied AFTER averaging over the group) or ``reinforce``
(``-A * sum log pi``), ``ratio_level`` ``sequence_mean`` | ``token``,
``kl_estimator`` ``logprob_diff`` | ``k3``.

B200-first changes: every prompt x G sample of a step is generated in one
batched call per prompt length (``RolloutEngine.rollout_many``; the reference
loops prompts one by one), and the old-policy log-probs recorded during the
rollout are reused instead of being recomputed by a second forward pass.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Any, Dict, List, Mapping, Optional, Sequence

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ConfigError
from rl_project_b200.core.protocols import RewardProvider, Trajectory
from rl_project_b200.rollouts.agent import AgentRolloutConfig, AgentRolloutEngine
from rl_project_b200.rollouts.engine import RolloutConfig, RolloutEngine, stack_group, stack_old_logprobs
from rl_project_b200.rollouts.rewards.composite import score_trajectories
from rl_project_b200.training.common.advantages import group_relative_advantages
from rl_project_b200.ops.rl_loss import clipped_kl_loss
from rl_project_b200.training.common.logprobs import (kl_k3, kl_logprob_diff, masked_mean, masked_sum,
                                                      packed_response_logprobs)
from rl_project_b200.training.common.trainer import PostTrainingAlgorithm
from rl_project_b200.training.ppo import ppo_clipped_objective


@dataclass
class GRPOConfig:
    group_size: int = 4
    prompts_per_step: int = 2
    clip_ratio: float = 0.2
    kl_coef: float = 0.04
    objective: str = "clipped"
    ratio_level: str = "sequence_mean"
    kl_estimator: str = "logprob_diff"
    advantage_eps: float = 1e-8
    skip_zero_variance_groups: bool = False
    agent: bool = False
    seed: int = 0

    def validate(self) -> None:
        if self.group_size < 2:
            raise ConfigError("GRPO group_size must be >= 2 (group-relative advantages need variance)")
        if self.objective not in ("clipped", "reinforce"):
            raise ConfigError("objective must be clipped|reinforce")
        if self.ratio_level not in ("sequence_mean", "token"):
            raise ConfigError("ratio_level must be sequence_mean|token")
        if self.kl_estimator not in ("logprob_diff", "k3"):
            raise ConfigError("kl_estimator must be logprob_diff|k3")


@dataclass
class GRPOGroup:
    trajectories: List[Trajectory]
    rewards: torch.Tensor
    advantages: torch.Tensor
    old_logprobs: Optional[torch.Tensor] = None
    ref_logprobs: Optional[torch.Tensor] = None
    skipped: bool = False


class GRPOAlgorithm(PostTrainingAlgorithm):
    name = "grpo"

    def __init__(self, policy, prompts, reward: RewardProvider, config: GRPOConfig,
                 rollout: Optional[RolloutConfig] = None, tasks: Optional[Sequence[Dict[str, Any]]] = None,
                 agent_rollout: Optional[AgentRolloutConfig] = None):
        config.validate()
        self.policy = policy
        self.cfg = config
        self.reward = reward
        self.rng = random.Random(config.seed)
        # the frozen reference only enters the clipped objective's KL term
        self._needs_ref = config.objective == "clipped" and config.kl_coef > 0
        if self._needs_ref and not policy.has_adapter and policy.reference_model is None:
            policy.with_frozen_reference()
        if config.agent:
            self.tasks = list(prompts)
            self.agent_engine = AgentRolloutEngine(policy, agent_rollout or AgentRolloutConfig())
            self.prompts: List[torch.Tensor] = []
        else:
            self.prompts = list(prompts)
            self.tasks = list(tasks) if tasks else [{} for _ in self.prompts]
            rc = rollout or RolloutConfig()
            rc.group_size = config.group_size
            self.rollouts = RolloutEngine(policy, rc)
        self._last_stats: Dict[str, float] = {}
        self._strategy: Any = None
        self._replica_set: Any = None
        self._shared_rng = random.Random(config.seed)  # identical on every rank: the replicas' prompt choice

    def bind_strategy(self, strategy: Any) -> None:
        """The distributed strategy the Trainer runs (rollout replicas read the learner's sharded weights)."""
        self._strategy = strategy

    def parameters(self) -> List[nn.Parameter]:
        return self.policy.trainable_parameters()

    def modules(self):
        return (self.policy.model,)

    def frozen_modules(self):
        return (self.policy.reference_model,) if self.policy.reference_model is not None else ()

    # ---------------------------------------------------------------- collection
    @torch.no_grad()
    def collect(self, step: int) -> List[GRPOGroup]:
        n = len(self.tasks if self.cfg.agent else self.prompts)
        if self.cfg.agent:
            idx = [self.rng.randrange(n) for _ in range(self.cfg.prompts_per_step)]
            # every episode of the step advances in one lock-step batch
            traj_groups = self.agent_engine.rollout_many([self.tasks[i] for i in idx], self.cfg.group_size)
        elif self.rollouts.cfg.replica_tp > 0 and torch.distributed.is_initialized():
            traj_groups = self._collect_replicated(step)
        else:
            idx = [self.rng.randrange(n) for _ in range(self.cfg.prompts_per_step)]
            traj_groups = self.rollouts.rollout_many([self.prompts[i] for i in idx], [self.tasks[i] for i in idx])
        groups, skipped = [], 0
        for trajs in traj_groups:
            rewards = torch.tensor(score_trajectories(self.reward, trajs), dtype=torch.float32)
            grp = GRPOGroup(trajs, rewards, group_relative_advantages(rewards, eps=self.cfg.advantage_eps))
            if self.cfg.skip_zero_variance_groups and float(rewards.std()) < 1e-6:
                grp.skipped = True
                skipped += 1
            elif self.cfg.objective == "clipped":
                self._attach_logprobs(grp)
            groups.append(grp)
        all_r = torch.cat([g.rewards for g in groups])
        n_traj = sum(len(g.trajectories) for g in groups)
        self._last_stats = {
            "reward_mean": float(all_r.mean()), "reward_std": float(all_r.std()) if all_r.numel() > 1 else 0.0,
            "group_std": float(torch.stack([g.rewards.std() for g in groups]).mean()),
            "groups_skipped": float(skipped),
            "response_len": float(sum(t.response_length for g in groups for t in g.trajectories) / max(1, n_traj)),
        }
        if self.cfg.agent:
            self._last_stats["tool_calls"] = float(sum(len(t.tool_results) for g in groups for t in g.trajectories))
        return groups

    @torch.no_grad()
    def _collect_replicated(self, step: int) -> List[List[Trajectory]]:
        """Every rank picks the same ``prompts_per_step`` prompts; each tensor-parallel replica generates its
        block of them (after taking the learner's current weights) and each rank keeps its share of the
        replica's groups, so the learner's per-rank batches need no exchange."""
        from rl_project_b200.inference.requests import SamplingParams
        from rl_project_b200.rollouts.engine import SEQ_ALIGN, _pad
        from rl_project_b200.rollouts.replicas import RolloutReplicas

        rc = self.rollouts.cfg
        if self._replica_set is None:
            dt = next(self.policy.model.parameters()).dtype
            self._replica_set = RolloutReplicas(self.policy.spec, rc.replica_tp, self.policy.device,
                                                dt if dt in (torch.bfloat16, torch.float16) else torch.float32,
                                                max_batch=rc.engine_max_batch, max_blocks=rc.engine_kv_blocks)
        rep = self._replica_set
        if self._strategy is not None and getattr(self._strategy, "units", None):
            rep.sync_from_fsdp(self._strategy)
        else:
            rep.sync_from_module(self.policy.model)
        chosen = [self._shared_rng.randrange(len(self.prompts)) for _ in range(self.cfg.prompts_per_step)]
        mine = rep.share(chosen)
        prompts = [self.prompts[i][-rc.max_prompt_length:].tolist() for i in mine]
        limit = rep.engine.max_seq_len
        G = self.cfg.group_size
        gens: List[List[List[int]]] = []
        for p in prompts:  # one request group per prompt: max tokens depend on the prompt length
            params = SamplingParams(max_tokens=max(1, min(rc.max_new_tokens, limit - len(p))),
                                    temperature=rc.temperature, top_k=rc.top_k, top_p=rc.top_p,
                                    stop_token_ids=[int(t) for t in rc.stop_token_ids])
            gens.append(params)
        outs = rep.generate_each(prompts, G, gens, seed=(self.cfg.seed * 1_000_003 + step) * 64 + rep.replica)
        dev = self.policy.device
        groups = []
        for j in rep.learner_share(list(range(len(mine)))):
            pid = torch.tensor(prompts[j], dtype=torch.long)
            rows = outs[j]
            responses = _pad(rows, dev, pid.numel(), SEQ_ALIGN)
            batch = pid.unsqueeze(0).repeat(G, 1).to(dev)
            old = self.rollouts._old_logprobs(batch, responses)  # one learner forward per group on every rank
            groups.append(self.rollouts._to_trajs(pid, responses, old, self.tasks[mine[j]], "",
                                                  lengths=[len(r) for r in rows]))
        return groups

    @torch.no_grad()
    def _attach_logprobs(self, grp: GRPOGroup) -> None:
        if self.cfg.agent:
            old = self.agent_engine.trajectories_logprob(grp.trajectories).float().cpu()
            ref = old
            if self._needs_ref:
                with self.policy.reference():
                    ref = self.agent_engine.trajectories_logprob(grp.trajectories).float().cpu()
            grp.old_logprobs, grp.ref_logprobs = old, ref
            return
        prompt, resp, mask = stack_group(grp.trajectories, self.policy.pad_token_id)
        if all(t.old_logprobs is not None for t in grp.trajectories):
            old = stack_old_logprobs(grp.trajectories, resp.shape[1]) * mask  # recorded at sampling time: same weights
        else:
            old = self.policy.logprobs(prompt, resp).float().cpu() * mask
        ref = old  # without a KL term the logged "kl" is the drift from the sampling policy
        if self._needs_ref:
            with self.policy.reference():
                ref = self.policy.logprobs(prompt, resp).float().cpu() * mask
        grp.old_logprobs, grp.ref_logprobs = old, ref

    # ---------------------------------------------------------------- objective
    def loss(self, groups: List[GRPOGroup], micro_step: int, n_micro: int):
        chunk = [g for g in (groups[micro_step::n_micro] if n_micro > 1 else groups) if not g.skipped]
        if not chunk:
            zero = sum(p.sum() for p in self.parameters()) * 0.0
            return zero, {**self._last_stats, "policy_loss": 0.0, "kl": 0.0}
        dev = self.policy.device
        news = [None] * len(chunk) if self.cfg.agent else self._packed_new(chunk)
        total = torch.zeros((), device=dev)
        kl_acc = torch.zeros((), device=dev)
        pl_acc = torch.zeros((), device=dev)
        for grp, new in zip(chunk, news):
            adv = grp.advantages.to(dev)
            if self.cfg.objective == "reinforce":
                loss, kl = self._reinforce_loss(grp, adv, new), torch.zeros((), device=dev)
            else:
                loss, kl = self._clipped_loss(grp, adv, new)
            total = total + loss
            pl_acc = pl_acc + loss.detach()
            kl_acc = kl_acc + kl.detach()
        n = len(chunk)
        return total / n, {**self._last_stats, "policy_loss": pl_acc / n, "kl": kl_acc / n}

    def _widths(self, grp: GRPOGroup) -> int:
        return grp.old_logprobs.shape[1] if grp.old_logprobs is not None else \
            max(t.response_length for t in grp.trajectories)

    def _packed_new(self, chunk: Sequence[GRPOGroup]) -> List[torch.Tensor]:
        """Every group's per-token log-probs ``[G, R_g]`` from ONE packed forward over all trajectories of the
        micro-batch (rows of different prompt lengths right-padded; exact under causal attention)."""
        trajs = [t for g in chunk for t in g.trajectories]
        widths = [self._widths(g) for g in chunk]
        lp, _ = packed_response_logprobs(self.policy, trajs, max(widths))
        out, row = [], 0
        for g, w in zip(chunk, widths):
            out.append(lp[row:row + len(g.trajectories), :w])
            row += len(g.trajectories)
        return out

    @staticmethod
    def _mask(grp: GRPOGroup, width: int, dev) -> torch.Tensor:
        lengths = torch.tensor([t.response_length for t in grp.trajectories], device=dev)
        return (torch.arange(width, device=dev)[None, :] < lengths[:, None]).float()

    def _kl(self, ref, new, mask):
        if self.cfg.kl_estimator == "k3":
            return kl_k3(ref, new, mask).mean()
        return kl_logprob_diff(ref, new, mask, clamp_min=None).mean().clamp(min=0)

    def _clipped_loss(self, grp: GRPOGroup, adv: torch.Tensor, new: Optional[torch.Tensor]):
        dev = self.policy.device
        if self.cfg.agent:
            new = self.agent_engine.trajectories_logprob(grp.trajectories).float()
            old, ref = grp.old_logprobs.to(dev), grp.ref_logprobs.to(dev)
            pl = ppo_clipped_objective(torch.exp(new - old), adv, self.cfg.clip_ratio).mean()
            kl = (ref - new).clamp(min=0).mean()
            return pl + self.cfg.kl_coef * kl, kl
        mask = self._mask(grp, new.shape[1], dev)
        old, ref = grp.old_logprobs.to(dev), grp.ref_logprobs.to(dev)
        # surrogate + KL (and their gradient) in one fused op; same formulas as _kl / ppo_clipped_objective
        loss, _, kl = clipped_kl_loss(new * mask, old, ref, mask, adv, self.cfg.clip_ratio, self.cfg.kl_coef,
                                      self.cfg.ratio_level, "k3" if self.cfg.kl_estimator == "k3" else "logprob_diff")
        return loss, kl

    def _reinforce_loss(self, grp: GRPOGroup, adv: torch.Tensor, new: Optional[torch.Tensor]) -> torch.Tensor:
        if self.cfg.agent:
            lp = self.agent_engine.trajectories_logprob(grp.trajectories).float()
            return (-adv * lp).sum()
        seq_lp = masked_sum(new, self._mask(grp, new.shape[1], self.policy.device))
        return (-adv * seq_lp).sum()

    # ---------------------------------------------------------------- evaluation
    @torch.no_grad()
    def evaluate(self, step: int) -> Dict[str, float]:
        """Greedy (agent) or sampled single completions of the first 8 prompts, decoded and scored as one batch."""
        n = min(8, len(self.tasks if self.cfg.agent else self.prompts))
        if n == 0:
            return {"reward": 0.0, "pass_rate": 0.0}
        if self.cfg.agent:
            groups = self.agent_engine.rollout_many(self.tasks[:n], 1, temperature=0.0)
        else:
            groups = self.rollouts.rollout_many(self.prompts[:n], self.tasks[:n], group_size=1)
        trajs = [t for g in groups for t in g]
        from rl_project_b200.rollouts.rewards.composite import batch_scores

        results = batch_scores(self.reward, trajs)
        return {"reward": sum(r.value for r in results) / max(len(results), 1),
                "pass_rate": sum(bool(r.passed) for r in results) / max(len(results), 1)}

    def state(self) -> Dict[str, Any]:
        return self.policy.state_for_checkpoint()

    def load_state(self, state: Mapping[str, Any]) -> None:
        self.policy.load_checkpoint_state(state)

    def model_spec(self) -> Dict[str, Any]:
        return self.policy.spec.to_dict()

    def tokenizer_meta(self):
        return self.policy.tokenizer.metadata()
