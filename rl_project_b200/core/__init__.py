"""Core: configuration, protocols, registry, runtime, lifecycle and errors."""

from rl_project_b200.core.config import (
    MODEL_PRESETS,
    AdapterConfig,
    CheckpointConfig,
    DataConfig,
    DistributedConfig,
    ExperimentManifest,
    ModelSpec,
    OptimizerConfig,
    PrecisionConfig,
    ScheduleConfig,
    TrainerConfig,
    load_config,
    model_spec_from_preset,
)
from rl_project_b200.core.errors import ForgelineError
from rl_project_b200.core.protocols import (
    EvaluationResult,
    GenerationSettings,
    PolicyModel,
    RewardProvider,
    RewardResult,
    Trajectory,
    Verifier,
)
from rl_project_b200.core.registry import Registry
from rl_project_b200.core.runtime import resolve_device, resolve_dtype, seed_everything


def __getattr__(name):  # RunContext imports observability; load it lazily to keep core import light
    if name in ("RunContext", "Stage"):
        from rl_project_b200.core import lifecycle

        return getattr(lifecycle, name)
    raise AttributeError(name)
