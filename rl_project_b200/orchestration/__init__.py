"""Optional worker orchestration (Ray) around the learner.

Nothing in the core imports Ray; ``rl_project_b200.orchestration.ray_backend``
raises ``OptionalDependencyError`` when Ray is missing.  Gradient and weight
traffic between GPUs stays on the ``parallel`` package (NCCL / NVLink kernels).
"""

from rl_project_b200.orchestration.config import (
    ORCHESTRATION_TYPES,
    RayConfig,
    orchestration_summary,
    ray_available,
    validate_orchestration,
)
