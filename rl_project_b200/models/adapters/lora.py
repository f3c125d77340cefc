"""Low-rank adapters: ``y = base(x) + scaling * (x A) B`` with ``scaling = alpha / rank`` (the capability of
``src/forgeline/models/adapters/lora.py``).

``A [in, rank]`` is Kaiming-uniform initialised and ``B [rank, out]`` zero, so a fresh adapter is the identity;
the parameter names (``lora_A``, ``lora_B``) and the state layout ``{module name: {lora_A, lora_B, rank, alpha}}``
are the checkpoint format of the reference, so adapter files carry over.

The adapter's contribution joins the base output inside one ``addmm`` (the rank-r product and the add share a
GEMM epilogue; no separate ``[tokens, out]`` delta tensor is written and re-read).  ``LoRALinear`` and the
quantised ``QLoRALinear`` share ``LowRankAdapter``; ``swap_linears`` is the one routine that replaces matching
``nn.Linear`` children, used to attach (``apply_lora``, ``apply_qlora``) and to merge (``merge_lora``).
"""

from __future__ import annotations

from typing import Callable, Dict, List, Optional, Sequence

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ModelError

DEFAULT_TARGET_MODULES: List[str] = ["q_proj", "k_proj", "v_proj", "c_proj", "wq", "wq_a", "wq_b", "wkv_a", "wkv_b",
                                     "wo", "w1", "w2", "w3", "c_fc"]


class LowRankAdapter(nn.Module):
    """The trainable low-rank pair around a frozen base layer (``self.base_forward``)."""

    def _init_adapter(self, in_features: int, out_features: int, rank: int, alpha: float, dropout: float,
                      device, dtype) -> None:
        if rank < 1:
            raise ModelError("LoRA rank must be >= 1")
        self.rank, self.alpha, self.scaling = rank, alpha, alpha / rank
        self.lora_A = nn.Parameter(nn.init.kaiming_uniform_(torch.empty(in_features, rank, device=device, dtype=dtype),
                                                            a=5 ** 0.5))
        self.lora_B = nn.Parameter(torch.zeros(rank, out_features, device=device, dtype=dtype))
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self.enabled = True

    def base_forward(self, x: torch.Tensor) -> torch.Tensor:  # pragma: no cover - overridden
        raise NotImplementedError

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        y = self.base_forward(x)
        if not self.enabled:
            return y
        lead = y.shape[:-1]
        low = self.dropout(x).reshape(-1, x.shape[-1]) @ self.lora_A.to(x.dtype)
        out = torch.addmm(y.reshape(-1, y.shape[-1]), low, self.lora_B.to(x.dtype), alpha=self.scaling)
        return out.view(*lead, out.shape[-1])


class LoRALinear(LowRankAdapter):
    def __init__(self, original: nn.Linear, rank: int, alpha: float = 16.0, dropout: float = 0.0):
        super().__init__()
        original.requires_grad_(False)
        self.original = original
        w = original.weight
        self._init_adapter(original.in_features, original.out_features, rank, alpha, dropout, w.device, w.dtype)

    @property
    def in_features(self) -> int:
        return self.original.in_features

    @property
    def out_features(self) -> int:
        return self.original.out_features

    def base_forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.original(x)

    def merge(self) -> nn.Linear:
        """Fold ``scaling * (A B)^T`` into the base weight and return the base layer."""
        with torch.no_grad():
            w = self.original.weight
            w.add_(((self.lora_A.float() @ self.lora_B.float()).t() * self.scaling).to(w.dtype))
        return self.original


def swap_linears(model: nn.Module, select: Callable[[str, nn.Module], bool],
                 make: Callable[[nn.Module], nn.Module]) -> int:
    """Replace every child ``c`` (attribute name ``attr``) with ``select(attr, c)`` by ``make(c)``; returns the count."""
    swaps = [(parent, attr, child) for parent in model.modules() for attr, child in parent.named_children()
             if select(attr, child)]
    for parent, attr, child in swaps:
        setattr(parent, attr, make(child))
    return len(swaps)


def attach_adapters(model: nn.Module, target_modules: Optional[Sequence[str]],
                    make: Callable[[nn.Linear], nn.Module]) -> nn.Module:
    """Freeze ``model`` and wrap every ``nn.Linear`` whose attribute name contains a target substring."""
    targets = list(target_modules) if target_modules else list(DEFAULT_TARGET_MODULES)
    model.requires_grad_(False)
    hits = swap_linears(model, lambda attr, c: isinstance(c, nn.Linear) and any(t in attr for t in targets), make)
    if not hits:
        raise ModelError(f"No linear layers matched target_modules={targets}")
    return model


def apply_lora(model: nn.Module, rank: int = 16, alpha: float = 32.0, dropout: float = 0.0,
               target_modules: Optional[Sequence[str]] = None) -> nn.Module:
    return attach_adapters(model, target_modules, lambda lin: LoRALinear(lin, rank, alpha, dropout))


def merge_lora(model: nn.Module) -> nn.Module:
    def unwrap(adapter: nn.Module) -> nn.Module:
        return adapter.merge().requires_grad_(True)

    swap_linears(model, lambda _attr, c: isinstance(c, LoRALinear), unwrap)
    return model


def _adapters(model: nn.Module) -> Dict[str, LowRankAdapter]:
    return {n: m for n, m in model.named_modules() if isinstance(m, LowRankAdapter)}


def set_lora_enabled(model: nn.Module, enabled: bool) -> None:
    for m in _adapters(model).values():
        m.enabled = enabled


def lora_state_dict(model: nn.Module) -> Dict[str, Dict[str, object]]:
    return {n: {"lora_A": m.lora_A.detach().clone(), "lora_B": m.lora_B.detach().clone(), "rank": m.rank,
                "alpha": m.alpha} for n, m in _adapters(model).items()}


def load_lora_state_dict(model: nn.Module, state: Dict[str, Dict[str, object]], strict: bool = True) -> int:
    live = _adapters(model)
    unknown = [n for n in state if n not in live]
    if unknown and strict:
        raise ModelError(f"LoRA state contains layer {unknown[0]!r} that the model does not have")
    loaded = 0
    for name in (n for n in state if n in live):
        entry, m = state[name], live[name]
        if m.rank != entry["rank"]:
            raise ModelError(f"LoRA rank mismatch for {name}: model {m.rank} vs state {entry['rank']}")
        with torch.no_grad():
            m.lora_A.copy_(entry["lora_A"])
            m.lora_B.copy_(entry["lora_B"])
        loaded += 1
    return loaded


def save_lora(model: nn.Module, path: str) -> int:
    state = lora_state_dict(model)
    torch.save(state, path)
    return sum(int(e["lora_A"].numel() + e["lora_B"].numel()) for e in state.values())


def load_lora(model: nn.Module, path: str, device: Optional[str] = None) -> int:
    return load_lora_state_dict(model, torch.load(path, map_location=device, weights_only=True))


def trainable_parameter_report(model: nn.Module) -> Dict[str, float]:
    counts = [(p.numel(), p.requires_grad) for p in model.parameters()]
    total = sum(n for n, _ in counts)
    train = sum(n for n, g in counts if g)
    return {"total": total, "trainable": train, "fraction": train / max(total, 1)}
