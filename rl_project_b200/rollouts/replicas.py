"""Tensor-parallel rollout replicas over the ranks of a distributed RL job.

The reference pushes the learner's full ``state_dict`` to Ray rollout workers through the object store
(``src/forgeline/orchestration/ray_backend.py:408-438``).  Here the ranks that train also generate:
``world / tp`` replicas of ``tp`` consecutive ranks each hold a tensor-parallel shard of a bf16 copy of the
policy (attention heads and FFN columns divided by ``tp``, all-reduce after the row-parallel projections,
embeddings and LM head replicated) and drive the paged-KV continuous-batching ``InferenceEngine`` over it.

* ``sync_from_fsdp`` / ``sync_from_module`` refresh the copy from the learner: each FSDP unit is gathered
  (a collective every rank takes, in unit order) and every rank copies its tensor-parallel slice of every
  parameter -- the slice is the ``rank``-th of ``tp`` equal chunks along the one dimension in which the
  shard's shape differs from the full parameter's (q/k/v/w1/w3 rows, o/w2 columns);
* ``generate`` runs one replica's prompts: its ``tp`` ranks submit the same requests in the same order and
  seed the engine's sampler identically, so after each layer's all-reduce their logits -- and hence every
  sampled token -- agree, and each rank returns the same completions;
* ``share`` splits a global list into the replicas' contiguous blocks (what a replica generates) and
  ``learner_share`` splits a replica's results over its ranks (what each rank trains on), so trajectories
  never move between ranks.
"""

from __future__ import annotations

from typing import Any, Iterable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from rl_project_b200.core.config import ModelSpec
from rl_project_b200.core.errors import DistributedConfigError


class RolloutReplicas:
    def __init__(self, spec: ModelSpec, tp_size: int, device: torch.device, dtype: torch.dtype = torch.bfloat16, *,
                 max_batch: int = 256, max_blocks: Optional[int] = None, timeout_s: Optional[float] = None):
        from rl_project_b200.inference.engine import InferenceEngine
        from rl_project_b200.models.transformer.model import TransformerLM
        from rl_project_b200.parallel.tensor_parallel import apply_tensor_parallel

        if not dist.is_initialized():
            raise DistributedConfigError("rollout replicas need an initialised process group")
        world, rank = dist.get_world_size(), dist.get_rank()
        if tp_size < 1 or world % tp_size:
            raise DistributedConfigError(f"rollout tensor_parallel {tp_size} must divide the world size {world}")
        self.tp, self.n_replicas = tp_size, world // tp_size
        self.replica, self.tp_rank = divmod(rank, tp_size)
        self.group = None
        kw = {}
        if timeout_s is not None:
            from datetime import timedelta

            kw["timeout"] = timedelta(seconds=timeout_s)
        if tp_size > 1:
            for r in range(self.n_replicas):  # every rank creates every group, in the same order
                g = dist.new_group(list(range(r * tp_size, (r + 1) * tp_size)), **kw)
                if r == self.replica:
                    self.group = g
        with torch.device(device):
            model = TransformerLM(spec)
        model = model.to(dtype).eval().requires_grad_(False)
        if tp_size > 1:
            apply_tensor_parallel(model, self.group, self.tp_rank, tp_size)
        self.model = model
        self._params = dict(model.named_parameters())
        per_seq = (spec.block_size + 15) // 16 + 1
        self.engine = InferenceEngine(model, max_batch=max_batch, max_blocks=max_blocks or max_batch * per_seq,
                                      decode_graphs=False)

    # ------------------------------------------------------------ weights
    @torch.no_grad()
    def load_full(self, name: str, full: torch.Tensor) -> None:
        """Copy this rank's slice of the full parameter ``name`` into the rollout copy (unknown names are skipped)."""
        dst = self._params.get(name)
        if dst is None:
            return
        src = full
        if tuple(src.shape) != tuple(dst.shape):
            dims = [i for i, (a, b) in enumerate(zip(src.shape, dst.shape)) if a != b]
            if len(dims) != 1 or src.shape[dims[0]] != dst.shape[dims[0]] * self.tp:
                raise DistributedConfigError(f"cannot slice {name} {tuple(src.shape)} into {tuple(dst.shape)}")
            src = src.chunk(self.tp, dims[0])[self.tp_rank]
        dst.copy_(src)

    def sync_from_module(self, module: nn.Module) -> None:
        for name, p in module.named_parameters():
            self.load_full(name, p.detach())

    def sync_from_fsdp(self, strategy: Any) -> None:
        """Gather every FSDP unit (a collective on every rank, in unit order) and take this rank's slices."""
        for u in strategy.units:
            was = u.gathered
            strategy.gather(u)
            for n, p in zip(u.names, u.params):
                self.load_full(f"{u.prefix}{n}", p.detach())
            if not was:
                u.free_full()

    # ------------------------------------------------------------ work split
    def share(self, items: Sequence[Any]) -> List[Any]:
        """This replica's contiguous block of ``items`` (the global list must divide evenly)."""
        n = len(items)
        if n % self.n_replicas:
            raise DistributedConfigError(f"{n} prompts do not divide over {self.n_replicas} rollout replicas")
        per = n // self.n_replicas
        return list(items[self.replica * per:(self.replica + 1) * per])

    def learner_share(self, items: Sequence[Any]) -> List[Any]:
        """This rank's block of its replica's results."""
        n = len(items)
        if n % self.tp:
            raise DistributedConfigError(f"{n} prompt groups do not divide over the replica's {self.tp} ranks")
        per = n // self.tp
        return list(items[self.tp_rank * per:(self.tp_rank + 1) * per])

    # ------------------------------------------------------------ generation
    @torch.no_grad()
    def generate(self, prompts: Sequence[Sequence[int]], group_size: int, params: Any,
                 seed: int) -> List[List[List[int]]]:
        """``group_size`` completions of every prompt (token lists), identical on every rank of the replica."""
        return self.generate_each(prompts, group_size, [params] * len(prompts), seed)

    @torch.no_grad()
    def generate_each(self, prompts: Sequence[Sequence[int]], group_size: int, params: Sequence[Any],
                      seed: int) -> List[List[List[int]]]:
        """As ``generate``, with sampling parameters per prompt."""
        from rl_project_b200.core.errors import RolloutError

        eng = self.engine
        with torch.random.fork_rng(devices=[]):  # the caller's host generator is left as it was
            torch.default_generator.manual_seed(seed)  # the engine draws its sampler seeds from this generator
            reqs = [[eng.submit(list(p), sp) for _ in range(group_size)] for p, sp in zip(prompts, params)]
            while not all(r.finished for grp in reqs for r in grp):
                eng.step()
        failed = [r for grp in reqs for r in grp if r.error]
        if failed:
            raise RolloutError(f"generation failed: {failed[0].error}")
        return [[list(r.generated_tokens) for r in grp] for grp in reqs]


def replica_layout(world: int, tp: int) -> List[Tuple[int, ...]]:
    """The ranks of every replica: consecutive blocks of ``tp`` (on one node: GPUs that share an NVSwitch domain)."""
    return [tuple(range(r * tp, (r + 1) * tp)) for r in range(world // tp)]
