"""Models and policies from specs and checkpoints (the contract of ``src/forgeline/models/loading.py``).

Every loader opens the checkpoint once (``_open``), resolves its model spec (a spec written by the reference
lacks this framework's additive fields, whose defaults reproduce the reference architecture), builds the
module directly on the target device (no CPU-side random init followed by a copy) and loads the weights.
Optional policy parts found in a checkpoint (LoRA adapter, value head) are restored through ``_POLICY_PARTS``.
"""

from __future__ import annotations

from pathlib import Path
from typing import Callable, Dict, Optional, Tuple

import torch

from rl_project_b200.checkpoints.manager import CheckpointManager, CheckpointState, load_model_state
from rl_project_b200.core.config import AdapterConfig, ModelSpec
from rl_project_b200.core.errors import CheckpointError, ModelError
from rl_project_b200.data.tokenizers import load_tokenizer, tokenizer_from_metadata
from rl_project_b200.models.policy import NativePolicy
from rl_project_b200.models.reward import SequenceRewardModel
from rl_project_b200.models.transformer.model import TransformerLM


def build_model(spec: ModelSpec, device: torch.device | str = "cpu") -> TransformerLM:
    with torch.device(device):
        return TransformerLM(spec)


def _open(path: str | Path, spec_override: Optional[ModelSpec] = None) -> Tuple[CheckpointState, ModelSpec]:
    state = CheckpointManager.load(path, map_location="cpu")
    if spec_override is not None:
        return state, spec_override
    if not state.model_spec:
        raise CheckpointError(f"checkpoint {path} has no model spec; pass spec_override")
    return state, ModelSpec.from_dict(dict(state.model_spec))


def _weights(state: CheckpointState) -> Dict[str, torch.Tensor]:
    """The model's own tensors: policy checkpoints nest them under ``model``, plain ones are flat."""
    ms = state.model_state
    return ms["model"] if "model" in ms else ms


def load_model_from_checkpoint(path: str | Path, device: torch.device | str = "cpu",
                               spec_override: Optional[ModelSpec] = None) -> Tuple[TransformerLM, ModelSpec, CheckpointState]:
    state, spec = _open(path, spec_override)
    model = build_model(spec, device)
    load_model_state(model, _weights(state), strict=False)
    return model.eval(), spec, state


def resolve_tokenizer_for_checkpoint(state: CheckpointState, data_dir: Optional[str | Path] = None):
    if state.tokenizer_meta:
        return tokenizer_from_metadata(state.tokenizer_meta)
    if data_dir is None:
        raise ModelError("checkpoint has no tokenizer metadata and no data_dir was given",
                         hint="Pass --data-dir pointing at the meta.pkl used for training.")
    return load_tokenizer(data_dir)


def _load_adapter(policy: NativePolicy, entry) -> None:
    if policy.has_adapter:
        from rl_project_b200.models.adapters.lora import load_lora_state_dict

        load_lora_state_dict(policy.model, entry, strict=False)


def _load_value_head(policy: NativePolicy, entry) -> None:
    if policy.value_head is not None:
        policy.value_head.load_state_dict(entry)


# checkpoint key -> how a policy takes it back
_POLICY_PARTS: Dict[str, Callable[[NativePolicy, object], None]] = {"adapter": _load_adapter,
                                                                    "value_head": _load_value_head}


def load_policy_from_checkpoint(path: str | Path, device: torch.device | str = "cpu",
                                data_dir: Optional[str | Path] = None, adapter: Optional[AdapterConfig] = None,
                                value_head: bool = False) -> NativePolicy:
    model, _, state = load_model_from_checkpoint(path, device)
    policy = NativePolicy(model, resolve_tokenizer_for_checkpoint(state, data_dir), adapter=adapter,
                          value_head=value_head)
    for key, restore in _POLICY_PARTS.items():
        if key in state.model_state:
            restore(policy, state.model_state[key])
    return policy.to(device)


def load_reward_model_from_checkpoint(path: str | Path, device: torch.device | str = "cpu") -> SequenceRewardModel:
    state, spec = _open(path)
    with torch.device(device):
        rm = SequenceRewardModel(spec, pooling=state.model_state.get("pooling", "last"))
    rm.load_state_dict(state.model_state["model"])
    return rm.eval()
