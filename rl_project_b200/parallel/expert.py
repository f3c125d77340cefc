"""Expert parallelism for MoE layers (strategy ``expert_parallel``).

The reference has none: every rank holds every expert and dispatch is a
Python mask loop.  Here the experts of each MoE layer are split over an
expert-parallel group of ``ep`` ranks (rank i keeps experts
``[i E/ep, (i+1) E/ep)``; the others become placeholders, so parameter names
stay global).  A forward:

1. routes locally and sorts the (token, slot) pairs by expert -- which also
   groups them by owning rank;
2. exchanges per-expert counts (``all_to_all_single`` of ``E`` integers), then
   the token rows (``all_to_all_single`` with the split sizes; autograd-aware,
   so the backward runs the reverse exchange);
3. regroups received rows by local expert, runs each local expert on its
   contiguous segment, restores the order and sends results back;
4. scatters the gate-weighted results into the token positions.

Non-expert parameters are replicated and averaged over all data-parallel
ranks; an expert's gradient already sums every rank's tokens (through the
all-to-all backward), so it is divided by the data-parallel width and summed
over the replicas that own the same expert (several EP groups).  The
aux-loss-free router bias is updated from global counts so it stays identical
on every rank.

On NCCL GPU ranks the exchange runs over NVLink peer memory instead
(parallel/expert_p2p.py: one gather kernel per exchange pulls rows straight
into the grouped-GEMM layout, no all-to-all and no re-permutation); the NCCL
all-to-all path below is the fallback (gloo, ``fused_comm`` off, buffers too
small).
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional

import torch
import torch.distributed as dist
import torch.distributed.nn.functional as dnnf
import torch.nn as nn

from rl_project_b200.core.config import DistributedConfig
from rl_project_b200.core.errors import DistributedConfigError
from rl_project_b200.parallel import runtime as rt
from rl_project_b200.parallel.data_parallel import _buckets


class _NoExpert(nn.Module):
    """Placeholder for an expert owned by another rank."""


def expert_parallel_moe(layer: nn.Module, xf: torch.Tensor, weights: torch.Tensor,
                        indices: torch.Tensor) -> torch.Tensor:
    from rl_project_b200.models.moe.layer import sort_by_expert
    from rl_project_b200.parallel import expert_p2p

    if expert_p2p.usable(layer, xf):  # peer-memory pulls straight into the grouped-GEMM layout
        out = expert_p2p.expert_parallel_moe_p2p(layer, xf, weights, indices)
        if out is not None:
            return out
    group = layer.expert_group
    ep = dist.get_world_size(group)
    E = layer.n_experts
    El = E // ep
    first = layer.local_experts[0]
    order, tok, counts = sort_by_expert(indices, E)
    xs = xf.index_select(0, tok)
    # per-expert counts: what I send to each rank -> what each rank sends me
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    both = torch.stack([counts.view(ep, El).sum(1), recv_counts.view(ep, El).sum(1)]).tolist()
    send_split, recv_split = both[0], both[1]
    rows = dnnf.all_to_all_single(xs.new_empty(sum(recv_split), xs.shape[1]), xs,
                                  output_split_sizes=recv_split, input_split_sizes=send_split, group=group)
    # received rows are grouped by source rank, then by local expert: regroup by local expert
    rc = recv_counts.view(ep, El)
    expert_of_row = torch.repeat_interleave(torch.arange(El, device=xf.device).repeat(ep), rc.reshape(-1))
    perm = torch.sort(expert_of_row, stable=True).indices
    local_counts = rc.sum(0).tolist()
    ys_sorted = layer.run_experts(rows.index_select(0, perm), local_counts, first_expert=first)
    ys_back = torch.empty_like(ys_sorted).index_copy(0, perm, ys_sorted)
    ys = dnnf.all_to_all_single(xs.new_empty(xs.shape[0], ys_back.shape[1]), ys_back,
                                output_split_sizes=send_split, input_split_sizes=recv_split, group=group)
    w = weights.reshape(-1).index_select(0, order).unsqueeze(-1).to(ys.dtype)
    return torch.zeros_like(xf).index_add_(0, tok, ys * w)


def shard_experts(layer: nn.Module, group: Any, rank_in_group: int, ep: int) -> None:
    if layer.n_experts % ep:
        raise DistributedConfigError(f"n_experts {layer.n_experts} not divisible by expert_parallel {ep}")
    El = layer.n_experts // ep
    lo = rank_in_group * El
    for e in range(layer.n_experts):
        if not lo <= e < lo + El:
            layer.experts[e] = _NoExpert()
        else:
            for p in layer.experts[e].parameters():
                p._expert_parallel = True
    layer.local_experts = list(range(lo, lo + El))
    layer.expert_group = group


class ExpertParallelStrategy:
    name = "expert_parallel"

    def __init__(self, cfg: DistributedConfig):
        self.cfg = cfg
        self.owns_grad_clip = True
        self.model: Optional[nn.Module] = None
        self.ep_group = None
        self.expert_dp_group = None

    def setup(self) -> None:
        rt.init_process_group(self.cfg.backend, timeout_s=self.cfg.timeout_s)
        world, rank, ep = rt.world_size(), rt.rank(), self.cfg.expert_parallel_size
        if ep < 2 or world % ep:
            raise DistributedConfigError(f"expert_parallel_size {ep} must be >= 2 and divide world size {world}")
        for lo in range(0, world, ep):  # EP groups: consecutive ranks
            g = dist.new_group(list(range(lo, lo + ep)))
            if lo <= rank < lo + ep:
                self.ep_group = g
        for i in range(ep):  # replicas of the same experts: same index in every EP group
            g = dist.new_group(list(range(i, world, ep)))
            if rank % ep == i:
                self.expert_dp_group = g
        from rl_project_b200.parallel import expert_p2p

        expert_p2p.set_enabled(getattr(self.cfg, "fused_comm", "auto") not in ("off", "nccl_baseline"))
        from rl_project_b200.parallel import health

        health.attach(self, self.cfg)

    def teardown(self) -> None:
        from rl_project_b200.parallel import expert_p2p

        if torch.cuda.is_available():
            torch.cuda.synchronize()
        expert_p2p.close_all()
        from rl_project_b200.parallel import health

        health.detach(self)
        rt.destroy_process_group()

    def check_health(self) -> None:
        if getattr(self, "monitor", None) is not None:
            self.monitor.check()

    def world_size(self) -> int:
        return rt.world_size()

    def rank(self) -> int:
        return rt.rank()

    def is_main_process(self) -> bool:
        return rt.rank() == 0

    def barrier(self) -> None:
        rt.barrier()

    def prepare_training(self, trainer) -> None:
        from rl_project_b200.models.moe.layer import MoELayer
        from rl_project_b200.parallel.mesh_strategies import _find_model

        model = _find_model(trainer.alg)
        ep = self.cfg.expert_parallel_size
        n = 0
        for blk in model.transformer.h:
            if isinstance(blk.ffn, MoELayer):
                shard_experts(blk.ffn, self.ep_group, rt.rank() % ep, ep)
                n += 1
        if n == 0:
            raise DistributedConfigError("expert_parallel needs a model with MoE layers")
        from rl_project_b200.models.moe.gate import share_router_counts

        share_router_counts([model], dist.group.WORLD)  # every rank routes its own tokens
        self.model = model
        from rl_project_b200.parallel.weight_sync import broadcast_parameters

        with torch.no_grad():  # replicated weights start identical; experts of each EP slot too
            for p in model.parameters():
                if getattr(p, "_expert_parallel", False) and self.cfg.expert_parallel_size < rt.world_size():
                    dist.broadcast(p.data, src=rt.rank() % ep, group=self.expert_dp_group)
        broadcast_parameters([p.data for p in model.parameters() if not getattr(p, "_expert_parallel", False)])

    def finish_gradients(self, trainer) -> None:
        world = rt.world_size()
        params = list(trainer.params)
        for p in params:
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        dense = [p for p in params if not getattr(p, "_expert_parallel", False)]
        expert = [p for p in params if getattr(p, "_expert_parallel", False)]
        for bucket in _buckets(dense, 256 << 20, lambda p: p.grad):
            self._reduce(bucket, 1.0 / world, None)
        if expert:
            replicas = world // self.cfg.expert_parallel_size
            for bucket in _buckets(expert, 256 << 20, lambda p: p.grad):
                self._reduce(bucket, 1.0 / world, self.expert_dp_group if replicas > 1 else "skip")

    @staticmethod
    def _reduce(bucket: List[torch.nn.Parameter], scale: float, group: Any) -> None:
        grads = [p.grad for p in bucket]
        flat = torch.cat([g.reshape(-1) for g in grads]) if len(grads) > 1 else grads[0].reshape(-1)
        flat.mul_(scale)
        if group != "skip":
            dist.all_reduce(flat, group=group)
        if len(grads) > 1:
            off = 0
            for g in grads:
                g.copy_(flat[off:off + g.numel()].view_as(g))
                off += g.numel()

    @torch.no_grad()
    def clip_grad_norm(self, params, max_norm: float, optimizer=None) -> torch.Tensor:
        params = [p for p in params if p.grad is not None]
        dev = params[0].device

        def sq(ps):
            if not ps:
                return torch.zeros((), device=dev)
            return torch.stack(torch._foreach_norm([p.grad.float() for p in ps])).pow(2).sum()

        dense = sq([p for p in params if not getattr(p, "_expert_parallel", False)])
        expert = sq([p for p in params if getattr(p, "_expert_parallel", False)])
        dist.all_reduce(expert, group=self.ep_group)  # experts are disjoint over the EP group
        norm = (dense + expert).sqrt()
        if max_norm > 0:
            if optimizer is not None and hasattr(optimizer, "arm_clip"):
                optimizer.arm_clip(norm, max_norm)
            else:
                coef = (max_norm / (norm + 1e-6)).clamp(max=1.0)
                coef = torch.where(torch.isfinite(norm), coef, torch.zeros_like(coef))
                torch._foreach_mul_([p.grad for p in params], coef)
        return norm

    def layout(self) -> Dict[str, Any]:
        return {"strategy": self.name, "world_size": rt.world_size(), "ep": self.cfg.expert_parallel_size}

    def sharded_checkpoint_state(self, trainer) -> Dict[str, Any]:
        from rl_project_b200.training.common.trainer import _cpu_state

        mine = _cpu_state(trainer._master_state(trainer.alg.state()))
        models: List[Any] = [None] * rt.world_size()
        opts: List[Any] = [None] * rt.world_size()
        dist.all_gather_object(models, mine)
        dist.all_gather_object(opts, trainer.optimizer.state_dict())
        return {"model": models, "optimizer": opts, "layout": self.layout()}

    def load_sharded_checkpoint_state(self, trainer, shards: Dict[str, Any]) -> None:
        if shards["layout"] != self.layout():
            raise DistributedConfigError(f"checkpoint layout {shards['layout']} does not match {self.layout()}")
        r = rt.rank()
        trainer.alg.load_state(shards["model"][r])
        if shards["optimizer"][r]:
            trainer.optimizer.load_state_dict(shards["optimizer"][r])
