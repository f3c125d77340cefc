"""Worker pools for rollouts, rewards, tools and sharded evaluation.

The pool logic is independent of where workers live: an ``ActorBackend``
spawns workers, submits method calls and waits on them.  ``ThreadBackend``
keeps each worker in this process with its own single-thread executor (calls
to one worker run in order, different workers run concurrently);
``rl_project_b200.orchestration.ray_backend`` provides Ray actors.

Recovery (the contract of ``src/forgeline/orchestration/ray_backend.py:181-318``):
every call remembers the generation of the worker it went to.  When a worker
is lost or a call times out, the worker is replaced once per generation, its
state is restored (constructor arguments plus, for rollout workers, the
latest weights) and the call is resubmitted, at most ``max_call_retries``
times.  Exceptions raised by user code inside a worker propagate unchanged.
"""

from __future__ import annotations

import concurrent.futures as cf
import copy
import os
import threading
import weakref
from typing import Any, Callable, Dict, List, Mapping, Optional, Sequence, Tuple

import torch

from rl_project_b200.core.errors import OrchestrationError
from rl_project_b200.core.protocols import EvaluationResult, RewardResult, Trajectory
from rl_project_b200.observability.logging import get_logger
from rl_project_b200.orchestration.config import RayConfig

log = get_logger("forgeline.orchestration")

_POOLS: "weakref.WeakSet[WorkerPool]" = weakref.WeakSet()


class WorkerLost(Exception):
    """A worker died or stopped answering: the call may be retried on a replacement."""


def chunks(items: Sequence[Any], n: int) -> List[List[Any]]:
    """Split into at most ``n`` contiguous, non-empty, near-equal parts."""
    n = max(1, min(n, len(items)))
    q, r = divmod(len(items), n)
    out, lo = [], 0
    for i in range(n):
        hi = lo + q + (1 if i < r else 0)
        out.append(list(items[lo:hi]))
        lo = hi
    return out


# ------------------------------------------------------------------ workers (plain classes, any backend)
class Worker:
    def __init__(self, torch_threads: int = 1):
        if torch_threads and os.environ.get("RLB_WORKER_SET_THREADS", "1") == "1":
            self._threads = torch_threads

    def pid(self) -> int:
        return os.getpid()

    def ping(self) -> bool:
        return True

    def device(self) -> str:
        return "cuda" if torch.cuda.is_available() else "cpu"


class RewardWorker(Worker):
    def __init__(self, reward: Any, torch_threads: int = 1):
        super().__init__(torch_threads)
        if isinstance(reward, Mapping):
            from rl_project_b200.rollouts.rewards import build_reward_provider

            reward = build_reward_provider(dict(reward))
        self.reward = reward

    def score(self, trajectories: List[Trajectory]) -> List[RewardResult]:
        many = getattr(self.reward, "score_many", None)
        return list(many(trajectories)) if many else [self.reward.score(t) for t in trajectories]


class ToolWorker(Worker):
    def execute(self, codes: List[str], timeout: float) -> List[Dict[str, Any]]:
        from rl_project_b200.rollouts.tools.python_executor import execute_python

        out = []
        for code in codes:
            r = execute_python(code, timeout=timeout)
            out.append({"output": r.output, "error": r.error, "timed_out": getattr(r, "timed_out", False)})
        return out


class RolloutWorker(Worker):
    """Holds its own copy of the policy model and samples with the in-process rollout engine."""

    def __init__(self, model: torch.nn.Module, tokenizer: Any, rollout_config: Any, seed: int, torch_threads: int = 1):
        super().__init__(torch_threads)
        from rl_project_b200.models.policy import NativePolicy
        from rl_project_b200.rollouts.engine import RolloutEngine

        self.policy = NativePolicy(model, tokenizer)
        self.engine = RolloutEngine(self.policy, rollout_config)
        self.version = -1
        self.gen = torch.Generator().manual_seed(seed)

    def load_weights(self, state: Dict[str, torch.Tensor], version: int) -> int:
        self.policy.model.load_state_dict(state)
        self.version = version
        return version

    def get_version(self) -> int:
        return self.version

    def rollout(self, prompt_ids: torch.Tensor, task: Optional[Dict[str, Any]], prompt_text: str,
                group_size: int) -> List[Trajectory]:
        return self.engine.rollout(prompt_ids, task, prompt_text, group_size=group_size)


class EvaluationWorker(Worker):
    def __init__(self, checkpoint: str, data_dir: Optional[str], torch_threads: int = 1):
        super().__init__(torch_threads)
        from rl_project_b200.core.runtime import resolve_device
        from rl_project_b200.models.loading import load_policy_from_checkpoint

        self.policy = load_policy_from_checkpoint(checkpoint, resolve_device("auto"), data_dir=data_dir)

    def run(self, benchmark: str, benchmark_kwargs: Dict[str, Any], indices: List[int],
            max_new_tokens: int) -> EvaluationResult:
        from rl_project_b200.evaluation.suites import BenchmarkSuite, build_benchmark

        suite = BenchmarkSuite(build_benchmark(benchmark, **benchmark_kwargs), max_new_tokens=max_new_tokens)
        return suite.run(self.policy, task_indices=indices)


# ------------------------------------------------------------------ backends
class ActorBackend:
    def spawn(self, cls: type, args: tuple, kwargs: dict, index: int, uses_gpu: bool) -> Any:
        raise NotImplementedError

    def submit(self, handle: Any, method: str, args: tuple) -> Any:
        raise NotImplementedError

    def wait_any(self, futures: List[Any], timeout: Optional[float]) -> Optional[Any]:
        raise NotImplementedError

    def result(self, future: Any) -> Any:
        raise NotImplementedError

    def kill(self, handle: Any) -> None:
        pass

    def put(self, obj: Any) -> Any:
        return obj


class _ThreadActor:
    def __init__(self, obj: Any):
        self.obj = obj
        self.pool = cf.ThreadPoolExecutor(max_workers=1)
        self.dead = False


class ThreadBackend(ActorBackend):
    """Workers as in-process objects; ``crash(handle)`` makes a worker's later calls fail as lost."""

    def spawn(self, cls, args, kwargs, index, uses_gpu):
        return _ThreadActor(cls(*args, **kwargs))

    def submit(self, handle: _ThreadActor, method: str, args: tuple):
        def run():
            if handle.dead:
                raise WorkerLost("worker is dead")
            return getattr(handle.obj, method)(*args)

        try:
            return handle.pool.submit(run)
        except RuntimeError as exc:  # executor shut down
            fut: cf.Future = cf.Future()
            fut.set_exception(WorkerLost(str(exc)))
            return fut

    def wait_any(self, futures, timeout):
        done, _ = cf.wait(futures, timeout=timeout, return_when=cf.FIRST_COMPLETED)
        return next(iter(done)) if done else None

    def result(self, future):
        return future.result()

    def kill(self, handle: _ThreadActor) -> None:
        handle.dead = True
        handle.pool.shutdown(wait=False, cancel_futures=True)

    @staticmethod
    def crash(handle: _ThreadActor) -> None:
        handle.dead = True


def make_backend(config: RayConfig) -> ActorBackend:
    if config.backend == "threads":
        return ThreadBackend()
    from rl_project_b200.orchestration.ray_backend import RayActorBackend

    return RayActorBackend(config)


# ------------------------------------------------------------------ pools
class WorkerPool:
    worker_class: type = Worker
    kind = "worker"
    uses_gpu = False

    def __init__(self, num_workers: int, config: Optional[RayConfig] = None, backend: Optional[ActorBackend] = None):
        if num_workers < 1:
            raise OrchestrationError(f"{self.kind} pool needs at least one worker")
        self.config = config or RayConfig()
        self.config.validate()
        self.backend = backend or make_backend(self.config)
        self.num_workers = num_workers
        self.restarts = 0
        self.workers: List[Any] = []
        self.generations: List[int] = []
        self._lock = threading.Lock()
        _POOLS.add(self)

    def _init_args(self, index: int) -> Tuple[tuple, dict]:
        return (), {"torch_threads": self.config.worker_torch_threads}

    def _restore(self, index: int) -> None:
        """Re-send state the constructor does not carry (e.g. the latest weights)."""

    def _spawn(self, index: int) -> Any:
        args, kwargs = self._init_args(index)
        return self.backend.spawn(self.worker_class, args, kwargs, index, self.uses_gpu)

    def _start(self) -> None:
        self.workers = [self._spawn(i) for i in range(self.num_workers)]
        self.generations = [0] * self.num_workers
        self.broadcast("ping")

    def _replace(self, index: int, generation: int, reason: BaseException) -> None:
        with self._lock:
            if self.generations[index] != generation:
                return  # already replaced after an earlier failure of the same worker
            self.backend.kill(self.workers[index])
            self.workers[index] = self._spawn(index)
            self.generations[index] += 1
            self.restarts += 1
        log.warning("worker_replaced", pool=self.kind, index=index, generation=self.generations[index],
                    reason=type(reason).__name__)
        self._restore(index)

    def call(self, calls: Sequence[Tuple[int, str, tuple]]) -> List[Any]:
        """Run ``(worker index, method, args)`` calls concurrently; results in call order."""
        def submit(j: int):
            w, m, a = calls[j]
            return w, self.generations[w], self.backend.submit(self.workers[w], m, a)

        pending = {j: submit(j) for j in range(len(calls))}
        attempts = [0] * len(calls)
        results: List[Any] = [None] * len(calls)
        recoverable = getattr(self.backend, "recoverable", (WorkerLost,))
        while pending:
            index = {id(f): j for j, (_, _, f) in pending.items()}
            done = self.backend.wait_any([f for _, _, f in pending.values()], self.config.task_timeout_s)
            if done is None:
                failed = {j: WorkerLost("task timeout") for j in pending}
            else:
                j = index[id(done)]
                try:
                    results[j] = self.backend.result(done)
                    pending.pop(j)
                    continue
                except recoverable as exc:
                    failed = {j: exc}
            for j, exc in failed.items():
                w, gen, _ = pending[j]
                attempts[j] += 1
                if attempts[j] > self.config.max_call_retries:
                    raise OrchestrationError(f"{self.kind} call {calls[j][1]!r} failed after {attempts[j]} attempts: "
                                             f"{type(exc).__name__}: {exc}")
                self._replace(w, gen, exc)
                pending[j] = submit(j)
        return results

    def broadcast(self, method: str, *args: Any) -> List[Any]:
        return self.call([(i, method, args) for i in range(self.num_workers)])

    def pids(self) -> List[int]:
        return self.broadcast("pid")

    def shutdown(self) -> None:
        for w in self.workers:
            try:
                self.backend.kill(w)
            except Exception:  # noqa: BLE001
                pass
        self.workers = []
        _POOLS.discard(self)

    def __enter__(self):
        return self

    def __exit__(self, *exc) -> None:
        self.shutdown()


class RewardPool(WorkerPool):
    """Scores trajectories in contiguous shards, one per worker (order preserved)."""

    worker_class, kind = RewardWorker, "reward"

    def __init__(self, reward: Any, num_workers: int, config: Optional[RayConfig] = None,
                 backend: Optional[ActorBackend] = None):
        super().__init__(num_workers, config, backend)
        self.reward_spec = reward
        inner = reward.get("type", "reward") if isinstance(reward, Mapping) else getattr(reward, "name", "reward")
        self.name = f"{inner}@pool"
        self._start()

    def _init_args(self, index):
        return (self.reward_spec,), {"torch_threads": self.config.worker_torch_threads}

    def score_many(self, trajectories: Sequence[Trajectory]) -> List[RewardResult]:
        if not trajectories:
            return []
        shards = chunks(list(trajectories), self.num_workers)
        return [r for part in self.call([(i, "score", (s,)) for i, s in enumerate(shards)]) for r in part]

    def score(self, trajectory: Trajectory) -> RewardResult:
        return self.score_many([trajectory])[0]


class ToolPool(WorkerPool):
    worker_class, kind = ToolWorker, "tool"

    def __init__(self, num_workers: int, config: Optional[RayConfig] = None, timeout: float = 5.0,
                 backend: Optional[ActorBackend] = None):
        super().__init__(num_workers, config, backend)
        self.timeout = timeout
        self._start()

    def execute_many(self, codes: Sequence[str]) -> List[Dict[str, Any]]:
        if not codes:
            return []
        shards = chunks(list(codes), self.num_workers)
        return [r for part in self.call([(i, "execute", (s, self.timeout)) for i, s in enumerate(shards)]) for r in part]


def weights_version(model: torch.nn.Module) -> int:
    """Sum of parameter version counters: changes whenever an optimiser step or load rewrites a parameter."""
    return int(sum(p._version for p in model.parameters()))


class RolloutPool(WorkerPool):
    """Drop-in ``RolloutEngine`` whose sampling runs in rollout workers; weights are pushed before a rollout
    whenever the learner's parameters changed since the last push (on-policy sampling)."""

    worker_class, kind, uses_gpu = RolloutWorker, "rollout", True

    def __init__(self, policy: Any, rollout_config: Any, num_workers: int, config: Optional[RayConfig] = None,
                 seed: int = 0, backend: Optional[ActorBackend] = None):
        if getattr(policy, "backend", "native") != "native":
            raise OrchestrationError("rollout workers support native policies",
                                     hint="Use in-process rollouts for the huggingface backend.")
        super().__init__(num_workers, config, backend)
        self.policy, self.cfg, self.seed = policy, rollout_config, seed
        self._model = self.backend.put(copy.deepcopy(policy.model).cpu())
        self._tokenizer = self.backend.put(policy.tokenizer)
        self._state = None
        self._version: Optional[int] = None
        self.weight_pushes = 0
        self._start()
        self.sync_weights(force=True)

    def _init_args(self, index):
        return ((self._model, self._tokenizer, self.cfg, self.seed + 1000 * index),
                {"torch_threads": self.config.worker_torch_threads})

    def _restore(self, index: int) -> None:
        if self._state is not None:
            self.backend.result(self.backend.submit(self.workers[index], "load_weights", (self._state, self._version)))

    def sync_weights(self, force: bool = False) -> bool:
        version = weights_version(self.policy.model)
        if not force and version == self._version:
            return False
        self._state = self.backend.put({k: v.detach().cpu().clone() for k, v in self.policy.model.state_dict().items()})
        self._version = version
        self.broadcast("load_weights", self._state, version)
        self.weight_pushes += 1
        return True

    def worker_versions(self) -> List[int]:
        return self.broadcast("get_version")

    def rollout(self, prompt_ids: torch.Tensor, task: Optional[Dict[str, Any]] = None, prompt_text: str = "",
                group_size: Optional[int] = None, temperature: Optional[float] = None) -> List[Trajectory]:
        self.sync_weights()
        G = group_size or self.cfg.group_size
        n = min(self.num_workers, G)
        counts = [G // n + (1 if i < G % n else 0) for i in range(n)]
        parts = self.call([(i, "rollout", (prompt_ids.cpu(), task, prompt_text, c)) for i, c in enumerate(counts)])
        return [t for part in parts for t in part]

    def rollout_many(self, prompts: Sequence[torch.Tensor], tasks: Optional[Sequence[Dict[str, Any]]] = None,
                     prompt_texts: Optional[Sequence[str]] = None,
                     group_size: Optional[int] = None) -> List[List[Trajectory]]:
        self.sync_weights()
        G = group_size or self.cfg.group_size
        return self.call([(i % self.num_workers, "rollout", (p.cpu(), tasks[i] if tasks else None,
                                                             prompt_texts[i] if prompt_texts else "", G))
                          for i, p in enumerate(prompts)])


class EvaluatorPool(WorkerPool):
    """Shards a benchmark's tasks over evaluation workers and merges per-item results exactly."""

    worker_class, kind, uses_gpu = EvaluationWorker, "evaluation", True

    def __init__(self, checkpoint: str, num_workers: int, config: Optional[RayConfig] = None,
                 data_dir: Optional[str] = None, backend: Optional[ActorBackend] = None):
        super().__init__(num_workers, config, backend)
        self.checkpoint, self.data_dir = str(checkpoint), data_dir
        self._start()

    def _init_args(self, index):
        return (self.checkpoint, self.data_dir), {"torch_threads": self.config.worker_torch_threads}

    def run(self, benchmark: str, max_new_tokens: int = 64, **benchmark_kwargs: Any) -> EvaluationResult:
        from rl_project_b200.evaluation.suites import build_benchmark

        n_tasks = len(build_benchmark(benchmark, **benchmark_kwargs).tasks())
        shards = chunks(list(range(n_tasks)), self.num_workers)
        parts: List[EvaluationResult] = self.call([(i, "run", (benchmark, benchmark_kwargs, s, max_new_tokens))
                                                   for i, s in enumerate(shards)])
        items = sorted((it for p in parts for it in p.per_item), key=lambda it: it["index"])
        correct = sum(bool(it["correct"]) for it in items)
        details = dict(parts[0].details) if parts else {}
        details.update({"workers": len(shards), "shard_sizes": [len(s) for s in shards]})
        return EvaluationResult(parts[0].suite if parts else f"benchmark/{benchmark}",
                                {"accuracy": correct / max(len(items), 1), "correct": float(correct)},
                                n_samples=len(items), details=details, per_item=items)


def shutdown_pools() -> None:
    for pool in list(_POOLS):
        pool.shutdown()


def attach_to_algorithm(algorithm: Any, orchestration: Mapping[str, Any], reward_config: Optional[Mapping[str, Any]],
                        seed: int = 0) -> Dict[str, Any]:
    """Swap an algorithm's in-process rollout engine / reward provider for worker pools per the manifest
    (algorithms exposing ``rollouts`` and ``reward``: PPO, GRPO, DAPO).  Agent-mode rollouts stay in process."""
    cfg = RayConfig.from_dict({k: v for k, v in orchestration.items() if k != "type"})
    attached: Dict[str, Any] = {"backend": cfg.backend}
    if cfg.reward_workers and hasattr(algorithm, "reward"):
        algorithm.reward = RewardPool(dict(reward_config) if reward_config else algorithm.reward, cfg.reward_workers,
                                      cfg)
        attached["reward_workers"] = cfg.reward_workers
    rollouts = getattr(algorithm, "rollouts", None)
    if cfg.rollout_workers and rollouts is not None and hasattr(algorithm, "policy"):
        algorithm.rollouts = RolloutPool(algorithm.policy, rollouts.cfg, cfg.rollout_workers, cfg, seed=seed)
        attached["rollout_workers"] = cfg.rollout_workers
    elif cfg.rollout_workers:
        attached["rollout_workers_skipped"] = f"{type(algorithm).__name__} has no single-turn rollout engine"
    log.info("orchestration_attached", **{k: str(v) for k, v in attached.items()})
    return attached
