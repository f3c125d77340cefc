"""Ray actors as the worker backend of the orchestration pools.

Importing this module requires Ray (``OptionalDependencyError`` otherwise).
``RayActorBackend`` runs each pool worker as a Ray actor (optionally inside a
placement group with one bundle per worker), waits with ``ray.wait`` and
classifies actor death / unavailability / timeouts as recoverable so the pool
replaces the worker and retries.  The ``Ray*`` pool names are the public names
of ``src/forgeline/orchestration/ray_backend.py``.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional

from rl_project_b200.core.errors import OptionalDependencyError, OrchestrationError
from rl_project_b200.orchestration.config import RayConfig
from rl_project_b200.orchestration import pools as _pools

try:
    import ray
    from ray.util.placement_group import placement_group, remove_placement_group
    from ray.util.scheduling_strategies import PlacementGroupSchedulingStrategy
except ImportError as exc:  # pragma: no cover - depends on the environment
    raise OptionalDependencyError("Ray orchestration requires Ray (pip install ray)",
                                  hint="Set orchestration.backend: threads to run workers in process.") from exc

_RECOVERABLE = tuple(t for t in (getattr(ray.exceptions, n, None) for n in
                                 ("RayActorError", "ActorUnavailableError", "WorkerCrashedError", "GetTimeoutError",
                                  "ObjectLostError")) if isinstance(t, type)) + (_pools.WorkerLost,)


def init_ray(config: Optional[RayConfig] = None) -> Dict[str, Any]:
    cfg = config or RayConfig()
    if not ray.is_initialized():
        kw: Dict[str, Any] = dict(ignore_reinit_error=True, include_dashboard=False, log_to_driver=False,
                                  namespace=cfg.namespace)
        if cfg.address is not None:
            kw["address"] = cfg.address
        else:
            if cfg.num_cpus is not None:
                kw["num_cpus"] = cfg.num_cpus
            if cfg.num_gpus is not None:
                kw["num_gpus"] = cfg.num_gpus
        ray.init(**kw)
    return dict(ray.cluster_resources())


def shutdown_ray() -> None:
    _pools.shutdown_pools()
    if ray.is_initialized():
        ray.shutdown()


shutdown_pools = _pools.shutdown_pools


class RayActorBackend(_pools.ActorBackend):
    recoverable = _RECOVERABLE

    def __init__(self, config: RayConfig):
        self.cfg = config
        init_ray(config)
        self._pg = None
        self._classes: Dict[type, Any] = {}

    def _placement(self, n_hint: int, uses_gpu: bool):
        if not self.cfg.placement_strategy or self._pg is not None:
            return self._pg
        bundle: Dict[str, float] = {"CPU": self.cfg.cpus_per_worker}
        if uses_gpu and self.cfg.gpus_per_worker:
            bundle["GPU"] = self.cfg.gpus_per_worker
        self._pg = placement_group([dict(bundle) for _ in range(n_hint)], strategy=self.cfg.placement_strategy)
        try:
            ray.get(self._pg.ready(), timeout=self.cfg.placement_timeout_s)
        except Exception as exc:  # noqa: BLE001
            remove_placement_group(self._pg)
            self._pg = None
            raise OrchestrationError(f"placement group {bundle} x {n_hint} could not be scheduled: "
                                     f"{type(exc).__name__}") from None
        return self._pg

    def spawn(self, cls, args, kwargs, index, uses_gpu):
        remote = self._classes.setdefault(cls, ray.remote(cls))
        opts: Dict[str, Any] = {"num_cpus": self.cfg.cpus_per_worker,
                                "num_gpus": self.cfg.gpus_per_worker if uses_gpu else 0,
                                "max_restarts": self.cfg.max_restarts}
        if self.cfg.memory_per_worker_mb:
            opts["memory"] = int(self.cfg.memory_per_worker_mb) << 20
        pg = self._placement(max(index + 1, self.cfg.rollout_workers, self.cfg.reward_workers, 1), uses_gpu)
        if pg is not None:
            opts["scheduling_strategy"] = PlacementGroupSchedulingStrategy(placement_group=pg,
                                                                           placement_group_bundle_index=index)
        return remote.options(**opts).remote(*args, **kwargs)

    def submit(self, handle, method, args):
        return getattr(handle, method).remote(*args)

    def wait_any(self, futures: List[Any], timeout):
        ready, _ = ray.wait(futures, num_returns=1, timeout=timeout)
        return ready[0] if ready else None

    def result(self, future):
        return ray.get(future)

    def kill(self, handle) -> None:
        try:
            ray.kill(handle, no_restart=True)
        except Exception:  # noqa: BLE001
            pass

    def put(self, obj: Any) -> Any:
        return ray.put(obj)


class _RayDefault:
    def __init__(self, *args, config: Optional[RayConfig] = None, **kwargs):
        cfg = config or RayConfig()
        super().__init__(*args, config=cfg, backend=RayActorBackend(cfg), **kwargs)  # type: ignore[call-arg]


class RayRewardPool(_RayDefault, _pools.RewardPool):
    pass


class RayToolPool(_RayDefault, _pools.ToolPool):
    pass


class RayRolloutEngine(_RayDefault, _pools.RolloutPool):
    pass


class RayEvaluator(_RayDefault, _pools.EvaluatorPool):
    pass


RewardWorker, ToolWorker, RolloutWorker, EvaluationWorker = (_pools.RewardWorker, _pools.ToolWorker,
                                                             _pools.RolloutWorker, _pools.EvaluationWorker)
attach_to_algorithm = _pools.attach_to_algorithm

__all__ = ["EvaluationWorker", "RayConfig", "RayEvaluator", "RayRewardPool", "RayRolloutEngine", "RayToolPool",
           "RewardWorker", "RolloutWorker", "ToolWorker", "attach_to_algorithm", "init_ray", "shutdown_pools",
           "shutdown_ray"]
