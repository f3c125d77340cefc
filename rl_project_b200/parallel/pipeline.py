"""Pipeline parallelism: contiguous block stages and a 1F1B schedule with a real backward.

``partition_model`` keeps on each stage only its contiguous slice of blocks
(the others become empty placeholders, so parameter names stay global and
checkpoints of all stages tile the full model); the first stage keeps the
embedding, the last the final norm and LM head (and, with tied embeddings, a
copy of the embedding whose gradient is summed with the first stage's).

``PipelineRunner`` drives ``n_micro`` micro-batches through the pipeline with
the 1F1B schedule: stage s runs ``min(P - s - 1, n_micro)`` warm-up forwards,
then alternates one forward / one backward, then drains the remaining
backwards.  Activations go forward and activation gradients go backward as
point-to-point messages, so every stage's parameters receive gradients --
unlike ``src/forgeline/distributed/pipeline_parallel.py``, whose scheduler ran
the backward on the last stage only.  Messages use the compute dtype (bf16 on
GPU).

Overlap: given one process group per direction of each stage pair (the mesh
builds them), the runner keeps ``lookahead`` receives posted in each
direction -- the activations of the next forwards and the gradients of the
next backwards -- so a transfer runs on the communicator's stream while the
stage computes the micro-batch before it; waiting on a receive makes the
compute stream wait, not the host.  Each directional group carries one
sender's messages in the order the receiver consumes them, which is what lets
receives be posted early (on a shared group, an early receive could be
matched ahead of a send the peer is blocked on).  Without directional groups
the runner posts each receive when it is needed, on the default group.

On NCCL the look-ahead defaults to 0 (each receive posted when it is consumed, still on its directional
group): in eager-init mode NCCL treats every unbatched send / receive as a collective of its communicator,
and with receives posted ahead a 2-stage 1F1B run deadlocked -- the first stage's host blocked posting a
gradient receive while the last stage's compute stream waited on an activation receive queued behind the
early ones.  ``RLB_PP_LOOKAHEAD`` overrides the depth; gloo keeps the default of 2.
"""

from __future__ import annotations

import os
from typing import Any, Callable, Dict, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist
import torch.nn as nn

from rl_project_b200.core.errors import DistributedConfigError


class _Placeholder(nn.Module):
    """Stands in for a block owned by another stage."""


def stage_bounds(n_layer: int, n_stages: int, stage: int) -> Tuple[int, int]:
    """Blocks ``[lo, hi)`` of ``stage``: near-equal contiguous slices, earlier stages take the remainder."""
    if n_stages > n_layer:
        raise DistributedConfigError(f"pipeline_parallel {n_stages} exceeds the {n_layer} layers")
    q, r = divmod(n_layer, n_stages)
    lo = stage * q + min(stage, r)
    return lo, lo + q + (1 if stage < r else 0)


def partition_model(model: nn.Module, stage: int, n_stages: int) -> nn.Module:
    """Drop the modules this stage does not own (in place)."""
    if n_stages == 1:
        return model
    L = len(model.transformer.h)
    lo, hi = stage_bounds(L, n_stages, stage)
    for i in range(L):
        if not lo <= i < hi:
            model.transformer.h[i] = _Placeholder()
    first, last = stage == 0, stage == n_stages - 1
    tied = model.lm_head.weight is model.transformer.wte.weight
    if not last:
        model.lm_head = None
        model.transformer.ln_f = _Placeholder()
        model.mtp_modules = None
    if not first and not (last and tied):
        model.transformer.wte = _Placeholder()
    if not first and getattr(model, "wpe", None) is not None:
        model.wpe = None
    model.pipeline_stage = (stage, n_stages, lo, hi)
    model.pipeline_tied = tied  # first and last stage then sum the embedding gradient
    return model


def stage_forward(model: nn.Module, x: torch.Tensor, first: bool) -> torch.Tensor:
    """Embedding (first stage) then this stage's blocks."""
    if first:
        x = model._embed(x)
    for blk in model.transformer.h:
        if not isinstance(blk, _Placeholder):
            x, _ = blk(x)
    return x


def stage_loss(model: nn.Module, h: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    from rl_project_b200.ops.logprob import linear_cross_entropy

    h = model.transformer.ln_f(h)
    return linear_cross_entropy(h.reshape(-1, h.shape[-1]), model.head_weight(), targets.reshape(-1))


def schedule_1f1b(n_micro: int, stage: int, n_stages: int) -> List[Tuple[str, int]]:
    """The ordered ("F" | "B", micro-batch) steps of one stage."""
    warm = min(n_stages - stage - 1, n_micro)
    steps = [("F", i) for i in range(warm)]
    for i in range(n_micro - warm):
        steps += [("F", warm + i), ("B", i)]
    steps += [("B", i) for i in range(n_micro - warm, n_micro)]
    return steps


_BATCHED = os.environ.get("RLB_PP_P2P", "plain") == "batched"


def _p2p(op, tensor: torch.Tensor, peer: int, tag: int, group: Any):
    """One point-to-point send / receive: plain ``isend`` / ``irecv``, or (``RLB_PP_P2P=batched``) a one-op
    ``batch_isend_irecv`` group (NCCL group semantics)."""
    if _BATCHED:
        return dist.batch_isend_irecv([dist.P2POp(op, tensor, peer, group=group, tag=tag)])[0]
    return op(tensor, peer, tag=tag, group=group)


def _backend(group: Any) -> str:
    if not dist.is_initialized():
        return ""
    try:
        return str(dist.get_backend(group))
    except (RuntimeError, ValueError):
        return ""


class _Inbox:
    """Receives of one direction, posted up to ``depth`` messages ahead in the order they will be consumed."""

    def __init__(self, src: Optional[int], group: Any, order: List[int], tag_of, depth: int):
        self.src, self.group, self.order, self.tag_of, self.depth = src, group, order, tag_of, depth
        self.posted: Dict[int, Tuple[torch.Tensor, Any]] = {}
        self.next = 0  # index into `order` of the next receive to post

    def _post(self, shape, dtype, device) -> None:
        i = self.order[self.next]
        self.next += 1
        buf = torch.empty(shape, dtype=dtype, device=device)
        self.posted[i] = (buf, _p2p(dist.irecv, buf, self.src, self.tag_of(i), self.group))

    def take(self, i: int, shape, dtype, device) -> torch.Tensor:
        while i not in self.posted:
            self._post(shape, dtype, device)
        buf, work = self.posted.pop(i)
        # keep `depth` receives in flight behind this one (they land while this micro-batch computes)
        while self.depth and self.next < len(self.order) and len(self.posted) < self.depth:
            self._post(shape, dtype, device)
        work.wait()  # NCCL: the compute stream waits for the transfer; gloo: the host waits
        return buf


class PipelineRunner:
    """Runs the 1F1B schedule of one stage for one optimiser step."""

    def __init__(self, model: nn.Module, stage: int, n_stages: int, prev_rank: Optional[int],
                 next_rank: Optional[int], group: Any = None, groups: Optional[Dict[str, Any]] = None,
                 lookahead: int = 2):
        self.model, self.stage, self.n_stages = model, stage, n_stages
        self.prev, self.next, self.group = prev_rank, next_rank, group
        self.first, self.last = stage == 0, stage == n_stages - 1
        g = groups or {}
        directional = all(g.get(k) is not None for k in
                          ([] if self.first else ["pp_act_in", "pp_grad_out"]) +
                          ([] if self.last else ["pp_act_out", "pp_grad_in"]))
        self.groups = g if directional else {}
        la = os.environ.get("RLB_PP_LOOKAHEAD")  # diagnostics / A-B: receives posted ahead (0: when needed)
        if la is not None:
            lookahead = int(la)
        elif _backend(group if group is not None else next(iter(self.groups.values()), None)) == "nccl":
            lookahead = 0
        self.lookahead = lookahead if directional else 0

    def _g(self, name: str):
        return self.groups.get(name, self.group)

    def run(self, micro_inputs: Sequence[Tuple[torch.Tensor, torch.Tensor]], act_shape: Tuple[int, ...],
            dtype: torch.dtype, device: torch.device, scale: float) -> torch.Tensor:
        """``micro_inputs[i] = (idx, targets)``; returns the summed scaled loss (last stage) or 0."""
        n = len(micro_inputs)
        steps = schedule_1f1b(n, self.stage, self.n_stages)
        acts = None if self.first else _Inbox(self.prev, self._g("pp_act_in"), [i for k, i in steps if k == "F"],
                                              lambda i: 2 * i, self.lookahead)
        grads = None if self.last else _Inbox(self.next, self._g("pp_grad_in"), [i for k, i in steps if k == "B"],
                                              lambda i: 2 * i + 1, self.lookahead)
        inputs: Dict[int, torch.Tensor] = {}
        outputs: Dict[int, torch.Tensor] = {}
        sends: List[Any] = []
        total = torch.zeros((), device=device, dtype=torch.float32)
        for kind, i in steps:
            if kind == "F":
                x_in = micro_inputs[i][0] if self.first else acts.take(i, act_shape, dtype, device).requires_grad_(True)
                out = stage_forward(self.model, x_in, self.first)
                if self.last:
                    loss = stage_loss(self.model, out, micro_inputs[i][1]) * scale
                    total += loss.detach().float()
                    outputs[i] = loss
                else:
                    sends.append(_p2p(dist.isend, out.detach().contiguous(), self.next, 2 * i, self._g("pp_act_out")))
                    outputs[i] = out
                inputs[i] = x_in
            else:
                out = outputs.pop(i)
                if self.last:
                    out.backward()
                else:
                    out.backward(grads.take(i, out.shape, out.dtype, device))
                x_in = inputs.pop(i)
                if not self.first:
                    sends.append(_p2p(dist.isend, x_in.grad.contiguous(), self.prev, 2 * i + 1, self._g("pp_grad_out")))
        for s in sends:
            s.wait()
        return total


# ---------------------------------------------------------------- reference-compatible names
# (src/forgeline/distributed/pipeline_parallel.py:16-110: PipelineStage, build_pipeline_stage,
# one_f_one_b_schedule, PipelineScheduler), built on the runner above -- which, unlike the reference's
# scheduler, also sends activation gradients back so every stage trains.

def one_f_one_b_schedule(n_micro: int, pp_rank: int, pp_size: int) -> List[Tuple[str, int]]:
    """The 1F1B action list of one rank: ``("F", i)`` / ``("B", i)`` over micro-batch indices."""
    return schedule_1f1b(n_micro, pp_rank, pp_size)


class PipelineStage(nn.Module):
    """This rank's slice of a ``TransformerLM`` (the whole model object, other stages' blocks replaced by
    placeholders): the first stage embeds, the last applies the final norm and the LM head."""

    def __init__(self, model: nn.Module, pp_rank: int, pp_size: int):
        super().__init__()
        self.model = partition_model(model, pp_rank, pp_size)
        self.pp_rank, self.pp_size = pp_rank, pp_size
        self.is_first, self.is_last = pp_rank == 0, pp_rank == pp_size - 1

    def forward(self, x: torch.Tensor, targets: Optional[torch.Tensor] = None):
        h = stage_forward(self.model, x, self.is_first)
        if self.is_last and targets is not None:
            return h, stage_loss(self.model, h, targets)
        return h, None


def build_pipeline_stage(model: nn.Module, mesh: Any) -> PipelineStage:
    """Stage ``mesh.pp_rank`` of ``mesh.pp_size`` (tensor-parallel sharding first when ``mesh.tp_size > 1``)."""
    if getattr(mesh, "tp_size", 1) > 1:
        from rl_project_b200.parallel.tensor_parallel import apply_tensor_parallel

        apply_tensor_parallel(model, mesh.groups.get("tp"), mesh.tp_rank, mesh.tp_size)
    return PipelineStage(model, mesh.pp_rank, mesh.pp_size)


class PipelineScheduler:
    """Runs 1F1B for one stage over ``n_micro`` chunks of a batch (forward and backward, activations and
    their gradients exchanged with the neighbouring stages); returns the summed loss on the last stage."""

    def __init__(self, stage: PipelineStage, mesh: Any, n_micro: int = 4):
        self.stage, self.mesh, self.n_micro = stage, mesh, n_micro
        self.runner = PipelineRunner(stage.model, mesh.pp_rank, mesh.pp_size, mesh.prev_stage, mesh.next_stage,
                                     groups=getattr(mesh, "groups", None))

    def run(self, inputs: torch.Tensor, targets: Optional[torch.Tensor] = None) -> torch.Tensor:
        if targets is None:
            raise ValueError("the pipeline schedule trains: targets are required")
        xs, ys = inputs.chunk(self.n_micro), targets.chunk(self.n_micro)
        model = self.stage.model
        dev = inputs.device
        dtype = next(p for p in model.parameters()).dtype
        act = (xs[0].shape[0], xs[0].shape[1], model.spec.n_embd)
        return self.runner.run(list(zip(xs, ys)), act, dtype, dev, 1.0 / self.n_micro)
