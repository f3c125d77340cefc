"""Process mesh for tensor x pipeline x data (x expert) parallelism.

Rank layout: ``rank = dp * (pp_size * tp_size) + pp * tp_size + tp`` -- tensor
parallel ranks are adjacent (the most communication-heavy groups stay on
consecutive GPUs of one NVSwitch node), then pipeline stages, then data
parallel replicas (the layout of ``src/forgeline/distributed/topology.py:13-74``,
so launch scripts place ranks the same way).  Every rank creates every group
in the same order, as ``torch.distributed.new_group`` requires.  Expert-parallel
groups partition the ``dp * tp`` ranks of one pipeline stage into groups of
``ep_size`` consecutive ranks.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import torch.distributed as dist

from rl_project_b200.core.errors import DistributedConfigError


@dataclass
class ParallelMesh:
    world_size: int
    tp_size: int = 1
    pp_size: int = 1
    ep_size: int = 1
    rank: int = 0
    groups: Dict[str, Any] = field(default_factory=dict)

    def __post_init__(self):
        if min(self.tp_size, self.pp_size, self.ep_size) < 1:
            raise DistributedConfigError("parallel degrees must be >= 1")
        if self.world_size % (self.tp_size * self.pp_size):
            raise DistributedConfigError(f"world_size {self.world_size} is not divisible by "
                                         f"tp {self.tp_size} x pp {self.pp_size}")
        if (self.dp_size * self.tp_size) % self.ep_size:
            raise DistributedConfigError(f"expert_parallel {self.ep_size} must divide dp*tp = "
                                         f"{self.dp_size * self.tp_size}")

    @property
    def dp_size(self) -> int:
        return self.world_size // (self.tp_size * self.pp_size)

    def coords(self, rank: Optional[int] = None) -> Dict[str, int]:
        r = self.rank if rank is None else rank
        per_dp = self.tp_size * self.pp_size
        return {"dp": r // per_dp, "pp": (r % per_dp) // self.tp_size, "tp": r % self.tp_size}

    def rank_of(self, dp: int, pp: int, tp: int) -> int:
        return dp * self.tp_size * self.pp_size + pp * self.tp_size + tp

    @property
    def tp_rank(self) -> int:
        return self.coords()["tp"]

    @property
    def pp_rank(self) -> int:
        return self.coords()["pp"]

    @property
    def dp_rank(self) -> int:
        return self.coords()["dp"]

    def tp_ranks(self, dp: Optional[int] = None, pp: Optional[int] = None) -> List[int]:
        c = self.coords()
        dp, pp = c["dp"] if dp is None else dp, c["pp"] if pp is None else pp
        return [self.rank_of(dp, pp, t) for t in range(self.tp_size)]

    def pp_ranks(self, dp: Optional[int] = None, tp: Optional[int] = None) -> List[int]:
        c = self.coords()
        dp, tp = c["dp"] if dp is None else dp, c["tp"] if tp is None else tp
        return [self.rank_of(dp, p, tp) for p in range(self.pp_size)]

    def dp_ranks(self, pp: Optional[int] = None, tp: Optional[int] = None) -> List[int]:
        c = self.coords()
        pp, tp = c["pp"] if pp is None else pp, c["tp"] if tp is None else tp
        return [self.rank_of(d, pp, tp) for d in range(self.dp_size)]

    def stage_ranks(self, pp: Optional[int] = None) -> List[int]:
        """All dp x tp ranks of one pipeline stage (the ranks expert parallelism spreads over)."""
        pp = self.coords()["pp"] if pp is None else pp
        return [self.rank_of(d, pp, t) for d in range(self.dp_size) for t in range(self.tp_size)]

    def ep_ranks(self) -> List[int]:
        stage = self.stage_ranks()
        i = stage.index(self.rank)
        lo = (i // self.ep_size) * self.ep_size
        return stage[lo:lo + self.ep_size]

    @property
    def prev_stage(self) -> Optional[int]:
        c = self.coords()
        return self.rank_of(c["dp"], c["pp"] - 1, c["tp"]) if c["pp"] > 0 else None

    @property
    def next_stage(self) -> Optional[int]:
        c = self.coords()
        return self.rank_of(c["dp"], c["pp"] + 1, c["tp"]) if c["pp"] < self.pp_size - 1 else None

    @property
    def is_first_stage(self) -> bool:
        return self.pp_rank == 0

    @property
    def is_last_stage(self) -> bool:
        return self.pp_rank == self.pp_size - 1

    def build_groups(self, timeout=None) -> "ParallelMesh":
        """Create tp / pp / dp / ep / embedding (first+last stage) groups; collective over all ranks."""
        if not dist.is_initialized():
            raise DistributedConfigError("torch.distributed must be initialised before building the mesh")
        kw = {"timeout": timeout} if timeout is not None else {}
        mine: Dict[str, Any] = {}

        def make(name: str, ranks: List[int]):
            g = dist.new_group(ranks, **kw)
            if self.rank in ranks:
                mine[name] = g

        for d in range(self.dp_size):
            for p in range(self.pp_size):
                make("tp", [self.rank_of(d, p, t) for t in range(self.tp_size)])
        for d in range(self.dp_size):
            for t in range(self.tp_size):
                ranks = [self.rank_of(d, p, t) for p in range(self.pp_size)]
                make("pp", ranks)
                make("embed", sorted({ranks[0], ranks[-1]}))
        # one two-rank group per direction of every adjacent stage pair: activations and activation gradients
        # then travel on separate communicators, each a single in-order stream, so a stage can post its
        # receives ahead of time without any ordering hazard against traffic in the other direction
        for d in range(self.dp_size):
            for t in range(self.tp_size):
                chain = [self.rank_of(d, p, t) for p in range(self.pp_size)]
                for a, b in zip(chain, chain[1:]):
                    acts, grads = dist.new_group([a, b], **kw), dist.new_group([a, b], **kw)
                    if self.rank == a:
                        mine["pp_act_out"], mine["pp_grad_in"] = acts, grads
                    if self.rank == b:
                        mine["pp_act_in"], mine["pp_grad_out"] = acts, grads
        for p in range(self.pp_size):
            for t in range(self.tp_size):
                make("dp", [self.rank_of(d, p, t) for d in range(self.dp_size)])
        for p in range(self.pp_size):
            stage = [self.rank_of(d, p, t) for d in range(self.dp_size) for t in range(self.tp_size)]
            for lo in range(0, len(stage), self.ep_size):
                make("ep", stage[lo:lo + self.ep_size])
        self.groups = mine
        return self

    def describe(self) -> Dict[str, Any]:
        return {"world_size": self.world_size, "tp": self.tp_size, "pp": self.pp_size, "dp": self.dp_size,
                "ep": self.ep_size, **{f"{k}_rank": v for k, v in self.coords().items()}}
