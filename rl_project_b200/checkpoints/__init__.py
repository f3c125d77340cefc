"""Atomic directory checkpoints with manifest validation and sharded extensions."""

from rl_project_b200.checkpoints.manager import CheckpointManager, CheckpointState, load_model_state
from rl_project_b200.checkpoints.validation import assert_compatible, compare_state_shapes, finite_state
