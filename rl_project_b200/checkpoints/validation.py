"""State-dict compatibility checks (``compare_state_shapes``, ``assert_compatible``, ``finite_state``)."""

from __future__ import annotations

from typing import Any, Dict, Mapping

import torch

from rl_project_b200.core.errors import IncompatibleStateError


def compare_state_shapes(model: torch.nn.Module, state: Mapping[str, Any]) -> Dict[str, Any]:
    own = model.state_dict()
    state = {k.replace("_orig_mod.", ""): v for k, v in state.items()}
    mismatched = {k: {"checkpoint": list(v.shape), "model": list(own[k].shape)} for k, v in state.items()
                  if k in own and isinstance(v, torch.Tensor) and v.shape != own[k].shape}
    return {"mismatched": mismatched, "missing": sorted(set(own) - set(state)),
            "unexpected": sorted(set(state) - set(own))}


def assert_compatible(model: torch.nn.Module, state: Mapping[str, Any]) -> None:
    rep = compare_state_shapes(model, state)
    if rep["mismatched"]:
        raise IncompatibleStateError(f"incompatible tensor shapes: {dict(list(rep['mismatched'].items())[:5])}")


def finite_state(state: Mapping[str, Any]) -> bool:
    for v in state.values():
        if isinstance(v, torch.Tensor) and v.is_floating_point() and not bool(torch.isfinite(v).all()):
            return False
        if isinstance(v, Mapping) and not finite_state(v):
            return False
    return True
