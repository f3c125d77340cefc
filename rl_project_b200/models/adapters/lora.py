"""Low-rank adapters ``y = W x + (x A B) * alpha / r`` (``src/forgeline/models/adapters/lora.py``).

``A [in, r]`` Kaiming-initialised, ``B [r, out]`` zero (identity at init);
``apply_lora`` matches child-module names against ``DEFAULT_TARGET_MODULES``
by substring and freezes everything else; state is ``{name: {lora_A, lora_B,
rank, alpha}}``.  Key names are the reference's so adapter checkpoints load.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ModelError

DEFAULT_TARGET_MODULES: List[str] = ["q_proj", "k_proj", "v_proj", "c_proj", "wq", "wq_a", "wq_b", "wkv_a", "wkv_b",
                                     "wo", "w1", "w2", "w3", "c_fc"]


class LoRALinear(nn.Module):
    def __init__(self, original: nn.Linear, rank: int, alpha: float = 16.0, dropout: float = 0.0):
        super().__init__()
        if rank < 1:
            raise ModelError("LoRA rank must be >= 1")
        self.original = original
        self.rank = rank
        self.alpha = alpha
        self.scaling = alpha / rank
        dev, dt = original.weight.device, original.weight.dtype
        self.lora_A = nn.Parameter(torch.empty(original.in_features, rank, device=dev, dtype=dt))
        self.lora_B = nn.Parameter(torch.zeros(rank, original.out_features, device=dev, dtype=dt))
        nn.init.kaiming_uniform_(self.lora_A, a=5 ** 0.5)
        original.weight.requires_grad = False
        if original.bias is not None:
            original.bias.requires_grad = False
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self.enabled = True

    @property
    def in_features(self) -> int:
        return self.original.in_features

    @property
    def out_features(self) -> int:
        return self.original.out_features

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.original(x)
        if not self.enabled:
            return y
        return y + (self.dropout(x) @ self.lora_A.to(x.dtype) @ self.lora_B.to(x.dtype)) * self.scaling

    def merge(self) -> nn.Linear:
        with torch.no_grad():
            delta = (self.lora_A.float() @ self.lora_B.float()).t() * self.scaling
            self.original.weight.add_(delta.to(self.original.weight.dtype))
        return self.original


def _children(model: nn.Module):
    for name, module in model.named_modules():
        for attr, child in list(module.named_children()):
            yield name, module, attr, child


def apply_lora(model: nn.Module, rank: int = 16, alpha: float = 32.0, dropout: float = 0.0,
               target_modules: Optional[Sequence[str]] = None) -> nn.Module:
    targets = list(target_modules) if target_modules else DEFAULT_TARGET_MODULES
    for p in model.parameters():
        p.requires_grad = False
    hit = 0
    for _, parent, attr, child in _children(model):
        if isinstance(child, nn.Linear) and any(t in attr for t in targets):
            setattr(parent, attr, LoRALinear(child, rank, alpha, dropout))
            hit += 1
    if not hit:
        raise ModelError(f"No linear layers matched target_modules={targets}")
    return model


def merge_lora(model: nn.Module) -> nn.Module:
    for _, parent, attr, child in _children(model):
        if isinstance(child, LoRALinear):
            lin = child.merge()
            lin.weight.requires_grad = True
            if lin.bias is not None:
                lin.bias.requires_grad = True
            setattr(parent, attr, lin)
    return model


def _is_adapter(m: nn.Module) -> bool:
    return hasattr(m, "lora_A") and hasattr(m, "lora_B") and hasattr(m, "enabled")


def set_lora_enabled(model: nn.Module, enabled: bool) -> None:
    for m in model.modules():
        if _is_adapter(m):
            m.enabled = enabled


def lora_state_dict(model: nn.Module) -> Dict[str, Dict[str, object]]:
    return {n: {"lora_A": m.lora_A.detach().clone(), "lora_B": m.lora_B.detach().clone(), "rank": m.rank,
                "alpha": m.alpha} for n, m in model.named_modules() if _is_adapter(m)}


def load_lora_state_dict(model: nn.Module, state: Dict[str, Dict[str, object]], strict: bool = True) -> int:
    mods = {n: m for n, m in model.named_modules() if _is_adapter(m)}
    n_loaded = 0
    for name, entry in state.items():
        if name not in mods:
            if strict:
                raise ModelError(f"LoRA state contains layer {name!r} that the model does not have")
            continue
        m = mods[name]
        if m.rank != entry["rank"]:
            raise ModelError(f"LoRA rank mismatch for {name}: model {m.rank} vs state {entry['rank']}")
        with torch.no_grad():
            m.lora_A.copy_(entry["lora_A"])
            m.lora_B.copy_(entry["lora_B"])
        n_loaded += 1
    return n_loaded


def save_lora(model: nn.Module, path: str) -> int:
    st = lora_state_dict(model)
    torch.save(st, path)
    return sum(int(s["lora_A"].numel() + s["lora_B"].numel()) for s in st.values())


def load_lora(model: nn.Module, path: str, device: Optional[str] = None) -> int:
    return load_lora_state_dict(model, torch.load(path, map_location=device, weights_only=True))


def trainable_parameter_report(model: nn.Module) -> Dict[str, float]:
    total = sum(p.numel() for p in model.parameters())
    train = sum(p.numel() for p in model.parameters() if p.requires_grad)
    return {"total": total, "trainable": train, "fraction": train / max(total, 1)}
