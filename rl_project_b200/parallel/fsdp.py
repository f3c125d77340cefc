"""Fully sharded data parallel (ZeRO-3) and ZeRO-2, written for this framework.

Layout.  Every trainable module is cut into *units*: one per transformer block
(``model.transformer.h[i]``) plus a root unit holding everything else
(embeddings, final norm, LM head, MTP heads).  A unit's parameters are laid
out back to back in one flat buffer padded to a multiple of ``world``; rank
``r`` owns the slice ``[r*S, (r+1)*S)`` as

* an fp32 master shard (the ``nn.Parameter`` the optimizer updates),
* a bf16 shard (what is all-gathered for compute),
* an fp32 gradient shard.

Forward: a pre-forward hook all-gathers the unit's bf16 shards into the full
flat buffer on a communication stream and points every parameter's ``.data``
at its slice; the gather of unit ``i+1`` is issued when unit ``i`` starts
(prefetch), so NCCL traffic overlaps compute.  With ``reshard_after_forward``
(the default) the full buffer's storage is released after the unit's forward and
re-gathered when its backward starts (the storage object is kept, so tensors
saved for backward stay valid); with it off, the gathered parameters stay
until the unit's gradients are reduced, trading memory for one all-gather per
unit and step.

Backward: when every parameter of a unit has accumulated its gradient
(``register_post_accumulate_grad_hook``), the gradients are packed into one
flat bf16 buffer and reduce-scattered on the communication stream straight
into the unit's fp32 gradient shard (averaged), then freed.  The root unit
(tied embedding/LM head gets gradients at both ends of backward) is reduced in
``finish_gradients``.

Optimizer: the fused sm_100a AdamW over the fp32 master shards writes the new
bf16 shard in the same pass.  Gradient clipping computes the squared norm of
the local shards on device, all-reduces one float, and finishes on device.

Checkpoint: every rank saves its own shards (``model.rank{r}.pt``,
``optimizer.rank{r}.pt``) with the unit layout in the manifest, so a run
resumes bit-for-bit without gathering a full state dict
(the reference gathers FULL_STATE_DICT to rank 0 and cannot resume FSDP:
``src/forgeline/training/common/trainer.py:243-253,293-297``).

On gloo (CPU tests) the same logic runs with all-gather / all-reduce
fallbacks for the collectives gloo lacks.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from rl_project_b200.core.config import DistributedConfig
from rl_project_b200.core.errors import DistributedConfigError
from rl_project_b200.parallel.strategies import _ProcessGroupStrategy


class _Unit:
    def __init__(self, name: str, module: nn.Module, params: List[Tuple[str, nn.Parameter]], world: int, rank: int,
                 device: torch.device, compute_dtype: torch.dtype, prefix: str = ""):
        self.name = name
        self.prefix = prefix
        self.module = module
        self.names = [n for n, _ in params]
        self.params = [p for _, p in params]
        self.shapes = [p.shape for p in self.params]
        self.numels = [p.numel() for p in self.params]
        self.offsets = []
        off = 0
        for n in self.numels:
            self.offsets.append(off)
            off += n
        self.total = off
        quantum = world * 8  # whole 16-byte vectors of bf16 per shard (fused reduce-scatter, vector loads)
        self.padded = (off + quantum - 1) // quantum * quantum
        self.shard = self.padded // world
        self.world, self.rank = world, rank
        self.device = device
        self.dtype = compute_dtype
        lo, hi = rank * self.shard, (rank + 1) * self.shard
        full32 = torch.zeros(self.padded, dtype=torch.float32, device=device)
        with torch.no_grad():
            for p, o, n in zip(self.params, self.offsets, self.numels):
                full32[o:o + n].copy_(p.detach().reshape(-1).float())
        self.master = nn.Parameter(full32[lo:hi].clone())
        self.master.fsdp_unit = self  # type: ignore[attr-defined]
        self.shard16 = self.master.detach().to(compute_dtype)
        self.full = full32.to(compute_dtype)  # every rank holds rank 0's weights here
        self._storage_bytes = self.full.untyped_storage().nbytes()
        self.gathered = False
        self.gather_event: Optional[torch.cuda.Event] = None
        self.pending_grads = 0
        self.rs_event = None
        self.grad_buf: Optional[torch.Tensor] = None  # persistent fp32 shard gradient (fused path)
        self.norm_counted = False  # the fused reduce added this unit's final gradient to the norm
        self._point_params_at_full()
        del full32

    # ---------------------------------------------------------------- parameter views
    def _point_params_at_full(self) -> None:
        for p, o, n, s in zip(self.params, self.offsets, self.numels, self.shapes):
            p.data = self.full[o:o + n].view(s)

    def free_full(self) -> None:
        if self.gathered:
            self.full.untyped_storage().resize_(0)
            self.gathered = False

    def ensure_storage(self) -> None:
        st = self.full.untyped_storage()
        if st.nbytes() != self._storage_bytes:
            st.resize_(self._storage_bytes)


class FSDPStrategy(_ProcessGroupStrategy):
    name = "fsdp"

    def __init__(self, cfg: DistributedConfig, reshard_params: bool = True, name: str = "fsdp"):
        super().__init__(cfg)
        self.name = name
        self.shard_params = reshard_params  # zero2 keeps full bf16 params between steps
        # False: a unit's gathered parameters stay until its backward (no re-gather; more memory)
        self.reshard_after_forward = bool(getattr(cfg, "reshard_after_forward", True))
        self.units: List[_Unit] = []
        self.root: Optional[_Unit] = None
        self.comm_stream = None
        self.group = None
        self._hooks: list = []
        self.fused = None  # FusedReduceScatter when gradients are reduced over peer memory
        self.fused_ag = None  # FusedAllGather when parameters are gathered over peer memory
        self.owns_grad_clip = False
        self._final_micro = True
        self._in_backward = True  # False inside finish_gradients
        self._rs_ctas_overlap = int(getattr(cfg, "fused_rs_ctas", 32))

    # ---------------------------------------------------------------- setup
    def _gloo(self) -> bool:
        return dist.get_backend(self.group) == "gloo"

    def prepare_training(self, trainer) -> None:
        if not dist.is_initialized():
            raise DistributedConfigError("call setup() before building the Trainer with an fsdp strategy")
        world, rank = dist.get_world_size(), dist.get_rank()
        device = trainer.ctx.device
        dtype = torch.bfloat16 if trainer.precision.master_weights else torch.float32
        mods = [m for m in trainer.alg.modules() if m is not None]
        if not mods:
            raise DistributedConfigError("fsdp needs the algorithm to expose its trained modules")
        # rank 0's initial weights everywhere (the same contract as DDP's broadcast)
        from rl_project_b200.parallel.weight_sync import broadcast_parameters

        broadcast_parameters([p.data for m in mods for p in m.parameters() if p.requires_grad], self.group)
        from rl_project_b200.models.moe.gate import share_router_counts

        share_router_counts(mods, self.group)  # MoE routers keep identical aux-free biases on every rank
        seen = set()
        for mi, m in enumerate(mods):
            blocks = list(m.transformer.h) if hasattr(m, "transformer") and hasattr(m.transformer, "h") else []
            for bi, blk in enumerate(blocks):
                ps = [(n, p) for n, p in blk.named_parameters() if p.requires_grad and id(p) not in seen]
                for _, p in ps:
                    seen.add(id(p))
                if ps:
                    self.units.append(_Unit(f"m{mi}.h{bi}", blk, ps, world, rank, device, dtype,
                                            prefix=f"transformer.h.{bi}."))
            rest = [(n, p) for n, p in m.named_parameters() if p.requires_grad and id(p) not in seen]
            for _, p in rest:
                seen.add(id(p))
            if rest:
                u = _Unit(f"m{mi}.root", m, rest, world, rank, device, dtype)
                self.units.append(u)
                self.root = u
        if device.type == "cuda":
            self.comm_stream = torch.cuda.Stream(device=device)
            self._setup_fused(device, dtype)
        for u in self.units:
            self._install_hooks(u)
        # params start gathered (full buffers hold the initial weights) -> release the block units
        if self.shard_params:
            for u in self.units:
                if u is not self.root:
                    u.gathered = True
                    u.free_full()
                else:
                    u.gathered = True
        else:
            for u in self.units:
                u.gathered = True

    def _setup_fused(self, device: torch.device, dtype: torch.dtype) -> None:
        """Reduce gradients with the fused peer-memory kernel (``fused_comm`` auto/on) when every rank is a GPU
        of this node on NCCL; ``off`` and ``nccl_baseline`` keep NCCL's reduce-scatter."""
        from rl_project_b200.parallel import fused_comm as fc

        mode = getattr(self.cfg, "fused_comm", "auto")
        world = dist.get_world_size(self.group)
        if mode in ("off", "nccl_baseline") or world == 1:
            return
        if mode == "auto" and world > 4:
            # measured: 2 ranks +2-3 % tokens/s over NCCL's reduce-scatter; 8 ranks -2.5 % (NCCL's NVLS
            # reduce-scatter overlaps backward with fewer SMs); `on` forces the fused path at any size
            return
        ok = fc.available(self.group) and dtype == torch.bfloat16
        if not ok:
            if mode == "on":
                raise DistributedConfigError("fused_comm=on needs bf16 gradients on NCCL ranks of one node")
            return
        # slots sized for the largest block unit; larger units (the root) go through in chunks
        blocks = [u for u in self.units if u is not self.root] or self.units
        chunk = max(u.shard for u in blocks)
        try:
            self.fused = fc.FusedReduceScatter(self.group, chunk * world, device,
                                               multicast=getattr(self.cfg, "fused_multicast", "off"),
                                               timeout_s=min(float(self.cfg.timeout_s), 300.0))
        except Exception as e:  # e.g. no peer mapping on this node: the same on every rank, before any collective
            if mode == "on":
                raise
            import warnings

            warnings.warn(f"fused reduce-scatter unavailable ({e}); using NCCL's")
            self.fused = None
            return
        for u in self.units:
            u.grad_buf = torch.zeros(u.shard, dtype=torch.float32, device=device)
        self.owns_grad_clip = True
        if mode == "on":  # parameter all-gather over peer memory too (opt-in)
            self.fused_ag = fc.FusedAllGather(self.group, max(u.shard for u in self.units), device,
                                              timeout_s=min(float(self.cfg.timeout_s), 300.0))

    # ---------------------------------------------------------------- collectives
    def _all_gather(self, u: _Unit) -> None:
        if u.gathered:
            return
        u.ensure_storage()
        if u.world == 1:
            u.full.copy_(u.shard16)
        elif self.fused_ag is not None:
            self.fused_ag.gather(u.shard16, u.full)
        elif self._gloo():
            parts = list(u.full.view(u.world, u.shard).unbind(0))
            dist.all_gather(parts, u.shard16)
        else:
            dist.all_gather_into_tensor(u.full, u.shard16)
        u.gathered = True

    def gather(self, u: _Unit, prefetch: bool = False) -> None:
        if u.gathered:
            if u.gather_event is not None and not prefetch:
                torch.cuda.current_stream().wait_event(u.gather_event)
                u.gather_event = None
            return
        if self.comm_stream is None:
            self._all_gather(u)
            return
        cur = torch.cuda.current_stream()
        self.comm_stream.wait_stream(cur)
        with torch.cuda.stream(self.comm_stream):
            self._all_gather(u)
            ev = torch.cuda.Event()
            ev.record(self.comm_stream)
        u.full.record_stream(self.comm_stream)
        u.gather_event = ev
        if not prefetch:
            cur.wait_event(ev)
            u.gather_event = None

    def _reduce_scatter(self, u: _Unit) -> None:
        grads = []
        for p, n in zip(u.params, u.numels):
            g = p.grad
            grads.append(g.reshape(-1) if g is not None else torch.zeros(n, dtype=u.dtype, device=u.device))
        if self.fused is not None:
            self._fused_reduce_scatter(u, grads)
            return
        pad = u.padded - u.total
        if pad:
            grads.append(torch.zeros(pad, dtype=grads[0].dtype, device=u.device))
        flat = torch.cat(grads)
        for p in u.params:
            p.grad = None

        def run():
            if u.world == 1:
                out = flat
            elif self._gloo():
                dist.all_reduce(flat, group=self.group)
                out = flat.view(u.world, u.shard)[u.rank]
            else:
                out = torch.empty(u.shard, dtype=flat.dtype, device=u.device)
                dist.reduce_scatter_tensor(out, flat, group=self.group)
            out = out.float().div_(u.world)
            if u.master.grad is None:
                u.master.grad = out
            else:
                u.master.grad.add_(out)

        if self.comm_stream is None:
            run()
            return
        self.comm_stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.comm_stream):
            run()
        flat.record_stream(self.comm_stream)

    def _fused_reduce_scatter(self, u: _Unit, grads: List[torch.Tensor]) -> None:
        """Pack the unit's bf16 gradients into symmetric slots and reduce the owned slice over peer memory into
        the persistent fp32 shard gradient (cast, 1/world, accumulation and squared norm in the same kernel)."""
        fr = self.fused
        cur = torch.cuda.current_stream()
        accumulate = u.master.grad is not None
        if not accumulate:
            u.master.grad = u.grad_buf
        norm = self._final_micro
        # reduces issued during backward share the SMs with it: a narrow grid (NCCL-like footprint);
        # the reduces issued after backward (finish_gradients) are on the critical path: the full grid
        ctas = self._rs_ctas_overlap if self._in_backward else 2 * torch.cuda.get_device_properties(
            u.device).multi_processor_count
        C = fr.slot_elems // u.world
        if u.shard <= C:
            slot = fr.next_slot(u.padded)
            torch.cat(grads, out=slot[:u.total])
            if u.padded > u.total:
                slot[u.total:].zero_()
            for p in u.params:
                p.grad = None
            self.comm_stream.wait_stream(cur)
            fr.reduce(u.shard, u.grad_buf, accumulate, norm, stream=self.comm_stream, ctas=ctas)
        else:
            flat = torch.cat(grads)
            if u.padded > u.total:
                flat = torch.cat([flat, flat.new_zeros(u.padded - u.total)])
            for p in u.params:
                p.grad = None
            rows = flat.view(u.world, u.shard)
            for c0 in range(0, u.shard, C):
                L = min(C, u.shard - c0)
                slot = fr.next_slot(u.world * L)
                slot.view(u.world, L).copy_(rows[:, c0:c0 + L])
                self.comm_stream.wait_stream(cur)
                fr.reduce(L, u.grad_buf[c0:c0 + L], accumulate, norm, stream=self.comm_stream, ctas=ctas)
            flat.record_stream(self.comm_stream)
        u.norm_counted = norm

    # ---------------------------------------------------------------- hooks
    def _install_hooks(self, u: _Unit) -> None:
        idx = self.units.index(u)

        def pre_forward(module, args):
            self.gather(u)
            if self.shard_params and idx + 1 < len(self.units) and self.units[idx + 1] is not self.root:
                self.gather(self.units[idx + 1], prefetch=True)
            return None

        def post_forward(module, args, output):
            if self.shard_params and u is not self.root and torch.is_grad_enabled():
                outs = output if isinstance(output, (tuple, list)) else (output,)
                # every differentiable output: whichever gradient arrives first re-gathers the unit
                for o in outs:
                    if isinstance(o, torch.Tensor) and o.requires_grad:
                        o.register_hook(lambda g, _u=u: self._pre_backward(_u, g))
                if self.reshard_after_forward:
                    self._release_after_forward(u)
            elif self.shard_params and u is not self.root:
                self._release_after_forward(u)
            return output

        def grad_ready(p):
            u.pending_grads -= 1
            if u.pending_grads == 0 and u is not self.root:
                self._reduce_scatter(u)
                if self.shard_params:
                    self._release_after_forward(u)

        if u is not self.root:
            self._hooks.append(u.module.register_forward_pre_hook(pre_forward))
            self._hooks.append(u.module.register_forward_hook(post_forward))
        for p in u.params:
            self._hooks.append(p.register_post_accumulate_grad_hook(grad_ready))

    def _release_after_forward(self, u: _Unit) -> None:
        if self.comm_stream is not None:
            u.full.record_stream(torch.cuda.current_stream())
        u.free_full()

    def _pre_backward(self, u: _Unit, grad):
        self.gather(u)
        idx = self.units.index(u)
        if idx > 0 and self.units[idx - 1] is not self.root:
            self.gather(self.units[idx - 1], prefetch=True)
        return grad

    # ---------------------------------------------------------------- trainer protocol
    def micro_step_context(self, micro: int, n_micro: int):
        from contextlib import nullcontext

        for u in self.units:
            u.pending_grads = len(u.params)
        self._final_micro = micro == n_micro - 1
        if self.fused is not None and micro == 0:
            self.fused.check()  # a timed-out wait of the previous step fails the run here
            self.fused.reset_norm()
            for u in self.units:
                u.norm_counted = False
        return nullcontext()

    def finish_gradients(self, trainer) -> None:
        self._in_backward = False
        if self.root is not None:
            self._reduce_scatter(self.root)
        for u in self.units:
            if u is not self.root and any(p.grad is not None for p in u.params):
                self._reduce_scatter(u)  # units whose hooks did not fire (unused params)
        self._in_backward = True
        if self.comm_stream is not None:
            torch.cuda.current_stream().wait_stream(self.comm_stream)
        for u in self.units:
            if u.master.grad is None:
                u.master.grad = torch.zeros_like(u.master)

    def build_optimizer(self, params, cfg):
        from rl_project_b200.training.common.optim import build_optimizer

        masters = [u.master for u in self.units]
        if masters[0].is_cuda and cfg.fused != "never":
            from rl_project_b200.ops.optim import FusedAdamW

            opt = FusedAdamW([{"params": masters, "weight_decay": cfg.weight_decay}], lr=cfg.learning_rate,
                             betas=(cfg.beta1, cfg.beta2), eps=cfg.eps, decoupled=(cfg.name == "adamw"),
                             param16={u.master: u.shard16 for u in self.units},
                             process_group=self.group if self.group is not None else dist.group.WORLD,
                             segments={u.master: self._segments(u, cfg) for u in self.units},
                             post_step=self.after_optimizer_step)
        else:
            opt = _ShardedTorchAdam(self, cfg)
        self.optimizer = opt
        return opt

    def _segments(self, u: _Unit, cfg):
        """(start, end, weight_decay) element ranges of the local shard, one per parameter it overlaps."""
        lo, hi = u.rank * u.shard, (u.rank + 1) * u.shard
        out = []
        for o, n, s in zip(u.offsets, u.numels, u.shapes):
            a, b = max(o, lo), min(o + n, hi)
            if a < b:
                wd = cfg.weight_decay if ((not cfg.decay_only_matrices) or len(s) >= 2) else 0.0
                out.append((a - lo, b - lo, wd))
        return out

    def _decay_mask(self, u: _Unit, cfg) -> torch.Tensor:
        """Per-element weight-decay multiplier over the unit's local shard (matrices only by default)."""
        full = torch.zeros(u.padded, dtype=torch.float32)
        for p, o, n, s in zip(u.params, u.offsets, u.numels, u.shapes):
            if (not cfg.decay_only_matrices) or len(s) >= 2:
                full[o:o + n] = 1.0
        return full[u.rank * u.shard:(u.rank + 1) * u.shard].to(u.device)

    def after_optimizer_step(self) -> None:
        for u in self.units:
            if not self.shard_params or u is self.root:
                # keep the full buffers current: re-gather the fresh bf16 shards
                u.gathered = False
                self.gather(u)

    def clip_grad_norm(self, params, max_norm: float, optimizer=None) -> torch.Tensor:
        if self.fused is not None:
            return self._fused_clip(max_norm, optimizer)
        sq = sum(u.master.grad.float().pow(2).sum() for u in self.units)
        dist.all_reduce(sq, group=self.group)
        norm = sq.sqrt()
        coef = (max_norm / (norm + 1e-6)).clamp(max=1.0)
        for u in self.units:
            u.master.grad.mul_(coef)
        return norm

    def _fused_clip(self, max_norm: float, optimizer) -> torch.Tensor:
        """Global gradient norm from the squares the fused reduce already summed (one float all-reduced); a
        rank whose reduce timed out contributes +inf, so every rank skips the update."""
        fr = self.fused
        sq = fr.sumsq.clone()
        for u in self.units:
            if not u.norm_counted:
                sq += u.master.grad.float().pow(2).sum()
        sq = torch.where(fr.status != 0, torch.full_like(sq, float("inf")), sq)
        fr.poll_status()
        dist.all_reduce(sq, group=self.group)
        norm = sq.sqrt()[0]
        if optimizer is not None and hasattr(optimizer, "arm_clip"):
            optimizer.arm_clip(norm, max_norm)
        elif max_norm > 0:
            coef = (max_norm / (norm + 1e-6)).clamp(max=1.0)
            coef = torch.where(torch.isfinite(norm), coef, torch.zeros_like(coef))
            for u in self.units:
                u.master.grad.mul_(coef)
        return norm

    def teardown(self) -> None:
        if self.fused is not None or self.fused_ag is not None:
            torch.cuda.synchronize()
        if self.fused is not None:
            self.fused.close()
            self.fused = None
        if self.fused_ag is not None:
            self.fused_ag.close()
            self.fused_ag = None
        super().teardown()

    # ---------------------------------------------------------------- checkpoints
    def layout(self) -> Dict[str, Any]:
        return {"world_size": dist.get_world_size(), "kind": self.name,
                "units": [{"name": u.name, "params": u.names, "shapes": [list(s) for s in u.shapes],
                           "offsets": u.offsets, "padded": u.padded, "shard": u.shard} for u in self.units]}

    def sharded_checkpoint_state(self, trainer) -> Dict[str, Any]:
        opt = trainer.optimizer
        mine = {"masters": [u.master.detach().cpu().clone() for u in self.units]}
        ostate = opt.state_dict()
        world = dist.get_world_size()
        models: List[Any] = [None] * world
        opts: List[Any] = [None] * world
        dist.all_gather_object(models, mine, group=self.group)
        dist.all_gather_object(opts, ostate, group=self.group)
        return {"model": models, "optimizer": opts, "layout": self.layout()}

    def load_sharded_checkpoint_state(self, trainer, shards: Dict[str, Any]) -> None:
        layout = shards["layout"]
        if int(layout["world_size"]) != dist.get_world_size():
            raise DistributedConfigError(
                f"checkpoint was sharded over {layout['world_size']} ranks, this run has {dist.get_world_size()}")
        r = dist.get_rank()
        mine = shards["model"][r]
        with torch.no_grad():
            for u, m in zip(self.units, mine["masters"]):
                u.master.copy_(m.to(u.device))
                u.shard16.copy_(u.master.to(u.dtype))
        if shards["optimizer"][r]:
            trainer.optimizer.load_state_dict(shards["optimizer"][r])
        for u in self.units:
            u.gathered = False
            if not self.shard_params or u is self.root:
                self.gather(u)

    def full_state_dict(self) -> Dict[str, torch.Tensor]:
        """Gather fp32 weights of every unit (collective); keys are the module's parameter names."""
        out: Dict[str, torch.Tensor] = {}
        for u in self.units:
            full = torch.empty(u.padded, dtype=torch.float32, device=u.device)
            if self._gloo():
                dist.all_gather(list(full.view(u.world, u.shard).unbind(0)), u.master.detach())
            else:
                dist.all_gather_into_tensor(full, u.master.detach())
            for n, o, k, s in zip(u.names, u.offsets, u.numels, u.shapes):
                out[f"{u.prefix}{n}"] = full[o:o + k].view(s).cpu()
        return out


class _ShardedTorchAdam(torch.optim.Optimizer):
    """CPU / non-fused path: torch AdamW on the fp32 master shards + bf16 shard refresh."""

    def __init__(self, strategy: FSDPStrategy, cfg):
        self.strategy = strategy
        masters = [u.master for u in strategy.units]
        cls = torch.optim.Adam if cfg.name == "adam" else torch.optim.AdamW
        self.inner = cls([{"params": masters, "weight_decay": 0.0}], lr=cfg.learning_rate,
                         betas=(cfg.beta1, cfg.beta2), eps=cfg.eps)
        self.wd = cfg.weight_decay
        self.masks = {u.master: strategy._decay_mask(u, cfg) for u in strategy.units}
        super().__init__(masters, {"lr": cfg.learning_rate})
        self.param_groups = self.inner.param_groups
        self.state = self.inner.state

    @torch.no_grad()
    def step(self, closure=None):
        lr = self.inner.param_groups[0]["lr"]
        for u in self.strategy.units:
            if self.wd:
                u.master.mul_(1 - lr * self.wd * self.masks[u.master])
        self.inner.step()
        for u in self.strategy.units:
            u.shard16.copy_(u.master.to(u.dtype))
        self.strategy.after_optimizer_step()

    def zero_grad(self, set_to_none: bool = True):
        self.inner.zero_grad(set_to_none=set_to_none)

    def state_dict(self):
        return self.inner.state_dict()

    def load_state_dict(self, sd):
        self.inner.load_state_dict(sd)
