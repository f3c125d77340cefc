"""The shared training lifecycle.

Contract: ``src/forgeline/training/common/trainer.py:32-325`` -- a
``PostTrainingAlgorithm`` owns data collection and the loss; ``Trainer``
owns the optimizer, learning-rate schedule, precision, gradient accumulation,
data-parallel gradient reduction, clipping, evaluation cadence, metrics and
checkpoint save/resume.

Design differences (B200-first):

* bf16 on CUDA trains bf16 parameters against fp32 master weights kept by the
  fused optimizer -- no autocast, no per-op casts.
* The step makes ONE host synchronisation: the loss, the metrics and the
  gradient norm are read together after the optimizer has been queued.  The
  global norm and the clip factor stay on the device.  A non-finite gradient
  makes the fused optimizer skip the update, and the non-finite loss is then
  reported as ``ConfigError`` exactly like the reference.
* Sharded strategies (FSDP/ZeRO) write per-rank checkpoint shards instead of
  gathering a full state dict to rank 0, so they can resume.
"""

from __future__ import annotations

import math
import os
import time
from abc import ABC, abstractmethod
from dataclasses import dataclass, field
from typing import Any, Dict, Iterable, List, Mapping, Optional, Tuple

import torch
import torch.nn as nn

from rl_project_b200.checkpoints.manager import CheckpointManager, CheckpointState
from rl_project_b200.core.config import TrainerConfig
from rl_project_b200.core.errors import CheckpointNotFoundError, ConfigError
from rl_project_b200.core.lifecycle import RunContext
from rl_project_b200.core.runtime import rng_state, set_rng_state
from rl_project_b200.observability.events import Event
from rl_project_b200.observability.metrics import device_memory_metrics, perf_metrics
from rl_project_b200.observability.tracing import nvtx_range
from rl_project_b200.training.common.optim import build_optimizer
from rl_project_b200.training.common.precision import Precision
from rl_project_b200.training.common.schedule import learning_rate_at


@dataclass
class StepResult:
    loss: float
    metrics: Dict[str, float] = field(default_factory=dict)


class PostTrainingAlgorithm(ABC):
    name: str = "algorithm"

    @abstractmethod
    def parameters(self) -> List[nn.Parameter]:
        ...

    @abstractmethod
    def collect(self, step: int) -> Any:
        ...

    @abstractmethod
    def loss(self, batch: Any, micro_step: int, n_micro: int):
        ...

    def modules(self) -> Iterable[nn.Module]:
        return ()

    def frozen_modules(self) -> Iterable[nn.Module]:
        """Modules used in the step but not trained (reference / teacher / reward models)."""
        return ()

    def cast_for_compute(self, dtype: torch.dtype) -> None:
        for m in list(self.modules()) + list(self.frozen_modules()):
            if m is not None:
                m.to(dtype)

    def evaluate(self, step: int) -> Dict[str, float]:
        return {}

    def state(self) -> Dict[str, Any]:
        return {}

    def load_state(self, state: Mapping[str, Any]) -> None:
        pass

    def model_spec(self) -> Dict[str, Any]:
        return {}

    def tokenizer_meta(self) -> Optional[Dict[str, Any]]:
        return None

    def on_step_end(self, step: int, result: StepResult) -> None:
        pass

    def tokens_in(self, batch: Any) -> int:
        """Tokens one step processes (the ``perf/*`` metrics).  Read from tensor shapes only, so it never
        synchronises: a tensor, or the first tensor of a tuple / list / dict batch; lists of groups of
        trajectories count prompt + response tokens.  0 when the batch says nothing (no perf metrics)."""
        if isinstance(batch, torch.Tensor):
            return int(batch.numel())
        if isinstance(batch, dict):
            batch = list(batch.values())
        if isinstance(batch, (list, tuple)) and batch:
            first = batch[0]
            if isinstance(first, torch.Tensor):
                return int(first.numel())
            trajs = [t for g in batch for t in (getattr(g, "trajectories", None) or [])]
            return sum(int(t.prompt_ids.numel()) + int(t.response_ids.numel()) for t in trajs
                       if hasattr(t, "prompt_ids") and hasattr(t, "response_ids"))
        return 0

    # data-position state, saved with every checkpoint so a resumed run draws the
    # same batches an uninterrupted run would (generators, shuffles, counters)
    _data_attrs = ("gen", "rng", "_order", "tokens_seen", "ema_loss")

    # the same kind of state on the algorithm's data source (``train`` / ``dataset``): a source that draws
    # from its own generator or walks its own cursor is restored too, saved as "<source>.<attr>"
    _source_names = ("train", "dataset", "sampler")
    _source_attrs = ("gen", "rng", "_order", "_i", "i", "pos", "_pos", "epoch")

    @staticmethod
    def _capture(val: Any):
        if isinstance(val, torch.Generator):
            return ("torch_gen", val.get_state())
        if hasattr(val, "getstate") and hasattr(val, "setstate"):
            return ("py_rng", val.getstate())
        if isinstance(val, (int, float, list, type(None))):
            return ("value", list(val) if isinstance(val, list) else val)
        return None

    def data_state(self) -> Dict[str, Any]:
        out: Dict[str, Any] = {}
        for name in self._data_attrs:
            if hasattr(self, name):
                c = self._capture(getattr(self, name))
                if c is not None:
                    out[name] = c
        for src_name in self._source_names:
            src = getattr(self, src_name, None)
            if src is None or isinstance(src, (torch.Tensor, list, tuple, dict)):
                continue
            for name in self._source_attrs:
                if hasattr(src, name):
                    c = self._capture(getattr(src, name))
                    if c is not None:
                        out[f"{src_name}.{name}"] = c
        return out

    def load_data_state(self, state: Mapping[str, Any]) -> None:
        for key, (kind, val) in (state or {}).items():
            obj, name = self, key
            if "." in key:
                src_name, name = key.split(".", 1)
                obj = getattr(self, src_name, None)
                if obj is None:
                    continue
            if kind == "torch_gen" and hasattr(obj, name):
                getattr(obj, name).set_state(val)
            elif kind == "py_rng" and hasattr(obj, name):
                getattr(obj, name).setstate(val)
            elif kind == "value":
                setattr(obj, name, list(val) if isinstance(val, list) else val)


def _as_tensor(v: Any, device: torch.device) -> torch.Tensor:
    if isinstance(v, torch.Tensor):
        return v.detach().float().reshape(()) if v.numel() == 1 else v.detach().float().mean()
    return torch.tensor(float(v), device=device)


def _cpu_state(obj: Any) -> Any:
    """Detached CPU copies of every tensor in a nested state."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu().clone()
    if isinstance(obj, dict):
        return {k: _cpu_state(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_cpu_state(v) for v in obj)
    return obj


class Trainer:
    def __init__(self, ctx: RunContext, algorithm: PostTrainingAlgorithm, config: Optional[TrainerConfig] = None,
                 checkpoint_manager: Optional[CheckpointManager] = None, strategy: Any = None):
        self.ctx = ctx
        self.alg = algorithm
        self.cfg = config or ctx.manifest.trainer
        self.cfg.validate()
        self.log = ctx.logger
        self.strategy = strategy
        self.precision = Precision(self.cfg.precision, ctx.device, ctx.dtype)
        if self.precision.master_weights:
            algorithm.cast_for_compute(torch.bfloat16)
        if self.cfg.gradient_checkpointing:
            for m in algorithm.modules():
                fn = getattr(m, "enable_gradient_checkpointing", None) or getattr(getattr(m, "model", None),
                                                                                  "enable_gradient_checkpointing", None)
                if fn:
                    fn()
        name = getattr(strategy, "name", "") if strategy is not None else ""
        world = strategy.world_size() if strategy is not None else 1
        self._sharded = name in ("fsdp", "zero2", "tensor_parallel", "pipeline_parallel", "hybrid",
                                 "expert_parallel") and world > 1
        self._sync_grads = name == "ddp" and world > 1
        # per-phase CUDA events of each step (forward, backward, grad_sync, clip, optimizer): off (None) unless a
        # caller sets a list, which train_step then appends (name, event) pairs to; recording costs no sync
        self.phase_events: Optional[List[Any]] = None
        if strategy is not None and hasattr(strategy, "prepare_training"):
            strategy.prepare_training(self)
        if strategy is not None and hasattr(algorithm, "bind_strategy"):
            algorithm.bind_strategy(strategy)
        self.params = [p for p in algorithm.parameters() if p.requires_grad]
        if not self.params:
            raise ConfigError("algorithm exposes no trainable parameters")
        if self._sync_grads:
            self._broadcast_parameters()
            from rl_project_b200.models.moe.gate import share_router_counts

            share_router_counts(getattr(self.alg, "modules", lambda: ())(), torch.distributed.group.WORLD)
        if self.cfg.compile_model:
            self._compile_modules()
        if strategy is not None and hasattr(strategy, "build_optimizer"):
            self.optimizer = strategy.build_optimizer(self.params, self.cfg.optimizer)
        else:
            self.optimizer = build_optimizer(self.params, self.cfg.optimizer, ctx.device)
        self.checkpoints = checkpoint_manager or CheckpointManager(
            ctx.output_dir / self.cfg.checkpoint.directory, keep_last=self.cfg.checkpoint.keep_last,
            async_save=self.cfg.checkpoint.async_save)
        self.step = 0
        self.best_metric: float = math.inf
        self.history: List[StepResult] = []
        self._tokens = 0  # tokens processed by this rank since the last perf log
        self._n_params = sum(p.numel() for p in self.params)

    # ------------------------------------------------------------ setup helpers
    def _compile_modules(self) -> None:
        names = []
        for m in self.alg.modules():
            if m is not None:
                m.compile(backend=self.cfg.compile_backend)
                names.append(type(m).__name__)
        self.log.info("compiled", backend=self.cfg.compile_backend, modules=",".join(names))

    def _broadcast_parameters(self) -> None:
        from rl_project_b200.parallel.data_parallel import broadcast_parameters

        broadcast_parameters(self.params, self.strategy)

    def _all_reduce_gradients(self) -> None:
        from rl_project_b200.parallel.data_parallel import all_reduce_gradients

        all_reduce_gradients(self.params, self.strategy)

    def current_lr(self) -> float:
        return learning_rate_at(self.step, self.cfg.optimizer.learning_rate, self.cfg.schedule)

    def _set_lr(self, lr: float) -> None:
        for g in self.optimizer.param_groups:
            g["lr"] = lr

    def _set_train_mode(self, mode: bool) -> None:
        for m in self.alg.modules():
            m.train(mode)

    # ------------------------------------------------------------ one optimizer step
    def _mark(self, name: str) -> None:
        if self.phase_events is not None and torch.cuda.is_available() and self.ctx.device.type == "cuda":
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.phase_events.append((name, ev))

    @staticmethod
    def phase_times(events: List[Any]) -> Dict[str, float]:
        """Milliseconds per phase from ``phase_events`` (synchronises): the time from each mark to the next is
        charged to the later mark's phase, summed over steps and micro-batches; ``start`` closes the gap
        between steps (batch collection, zero_grad)."""
        if not events:
            return {}
        events[-1][1].synchronize()
        out: Dict[str, float] = {}
        for (_, a), (name, b) in zip(events, events[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out

    def train_step(self) -> StepResult:
        if self.strategy is not None and hasattr(self.strategy, "check_health"):
            self.strategy.check_health()  # a dead peer fails here, before the step's first collective
        lr = self.current_lr()
        self._set_lr(lr)
        self._set_train_mode(True)
        batch = self.alg.collect(self.step)
        self._tokens += self.alg.tokens_in(batch)
        self.optimizer.zero_grad(set_to_none=True)
        self._mark("start")
        n_micro = self.cfg.gradient_accumulation_steps
        dev = self.ctx.device
        losses: List[torch.Tensor] = []
        metric_vals: Dict[str, List[torch.Tensor]] = {}
        scheduled = None
        if self.strategy is not None and hasattr(self.strategy, "run_micro_batches"):
            with self.precision.autocast():
                scheduled = self.strategy.run_micro_batches(self, batch, n_micro)  # e.g. a pipeline schedule
        if scheduled is not None:
            losses = [t.detach().float() for t in scheduled[0]]
            for k, v in scheduled[1].items():
                metric_vals.setdefault(k, []).append(_as_tensor(v, dev))
        for micro in range(n_micro if scheduled is None else 0):
            if self.strategy is not None and hasattr(self.strategy, "micro_step_context"):
                cm = self.strategy.micro_step_context(micro, n_micro)
            else:
                from contextlib import nullcontext

                cm = nullcontext()
            with cm, nvtx_range("rlb/forward_backward"):
                with self.precision.autocast():
                    loss, metrics = self.alg.loss(batch, micro, n_micro)
                self._mark("forward")
                if not loss.is_cuda and not bool(torch.isfinite(loss)):
                    raise ConfigError(f"non-finite loss at step {self.step}: {float(loss)}",
                                      hint="Lower the learning rate or check the reward / data pipeline.")
                self.precision.backward(loss / n_micro)
                self._mark("backward")
            losses.append(loss.detach().float())
            for k, v in metrics.items():
                metric_vals.setdefault(k, []).append(_as_tensor(v, dev))
        with nvtx_range("rlb/gradient_sync"):
            if self.strategy is not None and hasattr(self.strategy, "finish_gradients"):
                self.strategy.finish_gradients(self)
            elif self._sync_grads:
                self._all_reduce_gradients()
        self._mark("grad_sync")
        max_norm = self.cfg.optimizer.grad_clip
        norm_t: Optional[torch.Tensor] = None
        fused = hasattr(self.optimizer, "clip_grad_norm")
        if getattr(self.strategy, "owns_grad_clip", False):
            # norm over model-parallel shards, each parameter counted once
            self.precision.unscale(self.optimizer)
            norm_t = self.strategy.clip_grad_norm(self.params, max_norm, self.optimizer)
            fused = True
        elif fused:
            # fp16: the clip coefficient must see unscaled gradients (GradScaler then skips its own unscale)
            self.precision.unscale(self.optimizer)
            norm_t = self.optimizer.clip_grad_norm(max_norm if max_norm > 0 else 0.0)
        elif max_norm > 0:
            self.precision.unscale(self.optimizer)
            if self.strategy is not None and hasattr(self.strategy, "clip_grad_norm"):
                norm_t = self.strategy.clip_grad_norm(self.params, max_norm)
            else:
                norm_t = torch.nn.utils.clip_grad_norm_(self.params, max_norm)
        loss_mean = torch.stack(losses).mean() if len(losses) > 1 else losses[0]
        if not fused and not bool(torch.isfinite(loss_mean)):
            raise ConfigError(f"non-finite loss at step {self.step}: {float(loss_mean)}",
                              hint="Lower the learning rate or check the reward / data pipeline.")
        self._mark("clip")
        with nvtx_range("rlb/optimizer_step"):
            self.precision.step(self.optimizer)
        self._mark("optimizer")
        # the single host synchronisation of the step
        keys = sorted(metric_vals)
        packed = [loss_mean.to(dev)] + [torch.stack(metric_vals[k]).to(dev).mean() for k in keys]
        packed.append((norm_t.detach().float().to(dev) if norm_t is not None else torch.zeros((), device=dev)))
        vals = torch.stack([p.reshape(()) for p in packed]).tolist()
        total_loss, grad_norm = vals[0], vals[-1] if (max_norm > 0 or fused) else 0.0
        if not math.isfinite(total_loss):
            raise ConfigError(f"non-finite loss at step {self.step}: {total_loss}",
                              hint="Lower the learning rate or check the reward / data pipeline.")
        agg = {k: v for k, v in zip(keys, vals[1:-1])}
        agg.update({"lr": lr, "grad_norm": grad_norm if max_norm > 0 else 0.0})
        result = StepResult(loss=total_loss, metrics=agg)
        self.alg.on_step_end(self.step, result)
        self.step += 1
        self.history.append(result)
        return result

    # ------------------------------------------------------------ loop
    def fit(self, max_steps: Optional[int] = None) -> Dict[str, Any]:
        max_steps = self.cfg.max_steps if max_steps is None else max_steps
        self.ctx.metrics.event(Event.RUN_STARTED.value, {"algorithm": self.alg.name, "max_steps": max_steps})
        t0 = time.time()
        t_log, self._tokens = time.time(), 0
        last_eval: Dict[str, float] = {}
        try:
            while self.step < max_steps:
                if self.cfg.eval_every and self.step % self.cfg.eval_every == 0 and (self._is_main() or self._sharded):
                    last_eval = self._run_eval()
                if (self.cfg.checkpoint.save_every and self.step > 0
                        and self.step % self.cfg.checkpoint.save_every == 0):
                    self.save_checkpoint()
                result = self.train_step()
                log_step = bool(self.cfg.log_every) and self.step % self.cfg.log_every == 0
                if log_step:  # on every rank: the interval, its max over ranks (collective), the token count
                    now = time.time()
                    elapsed, tokens = now - t_log, self._tokens
                    # every rank reads its own index-error word; the code rides the same MAX all-reduce as
                    # the interval, so an out-of-range index skipped on any rank fails all ranks together
                    code = self._bounds_code()
                    slowest, code = self._slowest_rank_seconds(elapsed, code)
                    t_log, self._tokens = now, 0
                    if code:
                        from rl_project_b200.ops._ext import raise_bounds_error

                        raise_bounds_error(code)
                if log_step and self._is_main():
                    payload = {"train/loss": result.loss, **{f"train/{k}": v for k, v in result.metrics.items()}}
                    payload.update(device_memory_metrics(self.ctx.device))
                    # this rank's throughput since the last log (the step ends with one host sync, so the
                    # wall clock covers the device work); the data-parallel total is world x this
                    payload.update(perf_metrics(tokens, elapsed, self._n_params,
                                                float(os.environ.get("RLB_PEAK_TFLOPS", "0") or 0.0)))
                    if slowest is not None:
                        payload["perf/seconds_since_log_max_over_ranks"] = slowest
                    self.ctx.metrics.log(payload, step=self.step)
                    self.log.info("step", step=self.step, loss=round(result.loss, 5),
                                  **{k: round(v, 5) for k, v in result.metrics.items() if isinstance(v, float)})
            if self.cfg.eval_every and (self._is_main() or self._sharded):
                last_eval = self._run_eval()
            self.save_checkpoint(name="final")
            if self._is_main():
                self.checkpoints.wait()
        except BaseException as exc:
            self.ctx.metrics.event(Event.RUN_FAILED.value, {"error": repr(exc), "step": self.step})
            raise
        summary = {"steps": self.step, "elapsed_s": time.time() - t0,
                   "final_loss": self.history[-1].loss if self.history else None,
                   "best_metric": None if math.isinf(self.best_metric) else self.best_metric, "eval": last_eval}
        self.ctx.metrics.event(Event.RUN_FINISHED.value, summary)
        return summary

    def _bounds_code(self) -> int:
        """This rank's index-error word (read and cleared; 0 off CUDA or without the extension)."""
        if self.ctx.device.type != "cuda":
            return 0
        from rl_project_b200.ops._ext import available, bounds_code

        return bounds_code(self.ctx.device) if available() else 0

    def _slowest_rank_seconds(self, seconds: float, code: int = 0) -> Tuple[Optional[float], int]:
        """Max over ranks of (this rank's time since the last log, its index-error code): one collective
        every rank makes at log steps.  Single-process: ``(None, code)``."""
        if self.strategy is None or self.strategy.world_size() <= 1:
            return None, code
        import torch.distributed as dist

        if not dist.is_initialized():
            return None, code
        dev = self.ctx.device if dist.get_backend() == "nccl" else torch.device("cpu")
        t = torch.tensor([float(seconds), float(code)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        vals = t.tolist()
        return float(vals[0]), int(vals[1])

    def _is_main(self) -> bool:
        return self.strategy is None or self.strategy.is_main_process()

    def _run_eval(self) -> Dict[str, float]:
        self._set_train_mode(False)
        self.ctx.metrics.event(Event.EVAL_STARTED.value, {"step": self.step})
        with torch.no_grad():
            metrics = self.alg.evaluate(self.step)
        self._set_train_mode(True)
        if metrics and self._is_main():
            self.ctx.metrics.log({f"eval/{k}": v for k, v in metrics.items()}, step=self.step)
            self.log.info("eval", step=self.step, **{k: round(float(v), 5) for k, v in metrics.items()})
            primary = metrics.get("loss", metrics.get("primary"))
            if primary is not None and primary < self.best_metric and not self._sharded:
                self.best_metric = float(primary)
                self.save_checkpoint(name="best_candidate", is_best=True)
        self.ctx.metrics.event(Event.EVAL_FINISHED.value, {"step": self.step, **metrics})
        return metrics

    # ------------------------------------------------------------ checkpoints
    def _master_state(self, state: Any) -> Any:
        """Replace bf16 compute weights in ``state`` by their fp32 masters (bit-exact resume)."""
        masters = getattr(self.optimizer, "master_params", None)
        if masters is None:
            return state
        by_ptr = {p.data_ptr(): m for p, m in masters().items() if p.dtype != torch.float32}

        def swap(obj):
            if isinstance(obj, torch.Tensor):
                m = by_ptr.get(obj.data_ptr()) if obj.dtype == torch.bfloat16 else None
                return m.detach() if m is not None and m.shape == obj.shape else obj
            if isinstance(obj, dict):
                return {k: swap(v) for k, v in obj.items()}
            return obj

        return swap(state)

    def _rank_states(self) -> Optional[List[Dict[str, Any]]]:
        """Every rank's RNG and data-position state, gathered on every rank (collective).

        Data-parallel ranks draw different batches and samples; restoring the main rank's
        state on every rank would make a resumed run replay one stream on all of them."""
        if self.strategy is None or self.strategy.world_size() <= 1:
            return None
        import torch.distributed as dist

        if not dist.is_initialized():
            return None
        out: List[Any] = [None] * dist.get_world_size()
        dist.all_gather_object(out, {"rng": rng_state(), "data_state": self.alg.data_state()})
        return out

    def save_checkpoint(self, name: Optional[str] = None, is_best: bool = False):
        """Write a checkpoint.  Collective on every rank of a multi-rank run, except the
        ``is_best`` save, which only the main rank of an unsharded run makes."""
        ranks = None if is_best else self._rank_states()
        if self._sharded and hasattr(self.strategy, "sharded_checkpoint_state"):
            shards = self.strategy.sharded_checkpoint_state(self)
            if not self._is_main():
                self.strategy.barrier()
                return None
            state = CheckpointState(model_state={"sharded": True}, step=self.step, algorithm=self.alg.name,
                                    model_spec=self.alg.model_spec(), scaler_state=self.precision.state_dict(),
                                    rng_state=rng_state(),
                                    trainer_state={"best_metric": self.best_metric, "history_len": len(self.history),
                                                   "data_state": self.alg.data_state(), "rank_states": ranks},
                                    tokenizer_meta=self.alg.tokenizer_meta(), experiment=self.ctx.manifest.to_dict(),
                                    shards=shards)
            path = self.checkpoints.save(state, name=name, is_best=is_best)
            self.checkpoints.wait()
            self.strategy.barrier()
            self.ctx.metrics.event(Event.CHECKPOINT_SAVED.value, {"path": str(path), "step": self.step})
            return path
        if not self._is_main():
            return None
        model_state = self._master_state(self.alg.state())
        opt_state = self.optimizer.state_dict()
        state = CheckpointState(model_state=model_state, step=self.step, algorithm=self.alg.name,
                                model_spec=self.alg.model_spec(), optimizer_state=opt_state,
                                scaler_state=self.precision.state_dict(), rng_state=rng_state(),
                                trainer_state={"best_metric": self.best_metric, "history_len": len(self.history),
                                               "data_state": self.alg.data_state(), "rank_states": ranks},
                                tokenizer_meta=self.alg.tokenizer_meta(), experiment=self.ctx.manifest.to_dict())
        path = self.checkpoints.save(state, name=name, is_best=is_best)
        self.ctx.metrics.event(Event.CHECKPOINT_SAVED.value, {"path": str(path), "step": self.step})
        if name == "final" and self.cfg.adapter.merge_on_save:
            self._save_merged(state)
        return path

    def _save_merged(self, state: CheckpointState):
        import copy

        from rl_project_b200.models.adapters.lora import merge_lora

        policy = getattr(self.alg, "policy", None)
        if policy is None or not getattr(policy, "has_adapter", False) or not hasattr(policy.model, "spec"):
            self.log.warning("merge_on_save_skipped", reason="algorithm has no native policy with adapters")
            return None
        if self.cfg.adapter.method != "lora":
            self.log.warning("merge_on_save_skipped", reason=f"{self.cfg.adapter.method} base weights are quantized")
            return None
        merged = merge_lora(copy.deepcopy(policy.model)).float().state_dict()
        out = CheckpointState(model_state={"model": merged}, step=state.step, algorithm=state.algorithm,
                              model_spec=state.model_spec, tokenizer_meta=state.tokenizer_meta,
                              experiment=state.experiment, metadata={"merged_adapter": True})
        path = self.checkpoints.save(out, name="final_merged")
        self.ctx.metrics.event(Event.CHECKPOINT_SAVED.value, {"path": str(path), "step": self.step,
                                                              "merged_adapter": True})
        return path

    def resume(self, path: Optional[str] = None, strict_spec: bool = True) -> bool:
        target = path or self.cfg.checkpoint.resume_from or None
        if target is None:
            if not self.cfg.checkpoint.auto_resume:
                return False
            latest = self.checkpoints.find_latest()
            if latest is None:
                return False
            target = str(latest)
        expected = self.alg.model_spec() if strict_spec else None
        rank = self.strategy.rank() if self._sharded else None
        try:
            state = CheckpointManager.load(target, map_location="cpu", expected_spec=expected or None,
                                           expected_algorithm=self.alg.name, rank=rank)
        except CheckpointNotFoundError:
            if path or self.cfg.checkpoint.resume_from:
                raise
            return False
        if state.shards:
            self.strategy.load_sharded_checkpoint_state(self, state.shards)
        else:
            self.alg.load_state(state.model_state)
            if state.optimizer_state:
                self.optimizer.load_state_dict(state.optimizer_state)
            elif hasattr(self.optimizer, "load_state_dict") and hasattr(self.optimizer, "master_params"):
                # model-only checkpoint: masters start from the loaded weights
                with torch.no_grad():
                    for p, m in self.optimizer.master_params().items():
                        m.copy_(p.float())
        if state.scaler_state:
            self.precision.load_state_dict(state.scaler_state)
        ts = state.trainer_state or {}
        rng, data = state.rng_state, ts.get("data_state")
        ranks = ts.get("rank_states")
        if ranks and self.strategy is not None and len(ranks) == self.strategy.world_size():
            mine = ranks[self.strategy.rank()]  # this rank's own streams (same world size only)
            rng, data = mine["rng"], mine["data_state"]
        if rng:
            set_rng_state(rng)
        self.step = state.step
        self.best_metric = float(ts.get("best_metric", math.inf))
        if data:
            self.alg.load_data_state(data)
        self.ctx.metrics.event(Event.CHECKPOINT_LOADED.value, {"path": target, "step": self.step})
        self.log.info("resumed", path=target, step=self.step)
        return True
