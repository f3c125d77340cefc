"""Policies over the native transformer (``PolicyModel`` protocol).

``NativePolicy`` follows ``src/forgeline/models/policy.py:31-222``: LoRA /
QLoRA injection, reference = adapters disabled or a frozen copy,
per-token response log-probs, an optional value head, checkpoint dict
``{model, adapter, value_head}``.  Log-probs go through the fused LM-head
log-softmax kernel (ops/logprob.py), so no ``[B, T, V]`` fp32 tensor is
built.  ``HFPolicy`` lives in models/hf_policy.py (optional dependency).
"""

from __future__ import annotations

import copy
from contextlib import contextmanager
from typing import Any, Dict, Iterator, List, Mapping, Optional

import torch
import torch.nn as nn

from rl_project_b200.core.config import AdapterConfig, ModelSpec
from rl_project_b200.core.errors import ConfigError, ModelError
from rl_project_b200.core.protocols import GenerationSettings
from rl_project_b200.models.adapters.lora import apply_lora, load_lora_state_dict, lora_state_dict, set_lora_enabled
from rl_project_b200.models.adapters.qlora import apply_qlora
from rl_project_b200.models.generation.sampling import generate_tokens
from rl_project_b200.models.transformer.model import TransformerLM
from rl_project_b200.ops.logprob import linear_logprobs, logprobs_from_logits


class ValueHead(nn.Module):
    def __init__(self, hidden_size: int, dropout: float = 0.1):
        super().__init__()
        self.net = nn.Sequential(nn.Dropout(dropout), nn.Linear(hidden_size, hidden_size // 2), nn.GELU(),
                                 nn.Linear(hidden_size // 2, 1))

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.net(hidden.to(self.net[1].weight.dtype)).squeeze(-1)


def token_logprobs_from_logits(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    return logprobs_from_logits(logits, labels)


class NativePolicy(nn.Module):
    backend = "native"

    def __init__(self, model: TransformerLM, tokenizer: Any, *, pad_token_id: int = 0,
                 adapter: Optional[AdapterConfig] = None, reference_model: Optional[TransformerLM] = None,
                 value_head: bool = False):
        super().__init__()
        self.model = model
        self.tokenizer = tokenizer
        self.pad_token_id = pad_token_id
        self.spec: ModelSpec = model.spec
        self.adapter = adapter or AdapterConfig()
        self._has_adapter = self.adapter.method in ("lora", "qlora")
        if self.adapter.method == "lora":
            apply_lora(model, self.adapter.rank, self.adapter.alpha, self.adapter.dropout,
                       self.adapter.target_modules or None)
        elif self.adapter.method == "qlora":
            apply_qlora(model, self.adapter.rank, self.adapter.alpha, self.adapter.dropout,
                        self.adapter.target_modules or None)
        self.reference_model = reference_model
        self.value_head: Optional[ValueHead] = ValueHead(self.spec.n_embd) if value_head else None

    @classmethod
    def from_spec(cls, spec: ModelSpec, tokenizer: Any, **kw: Any) -> "NativePolicy":
        return cls(TransformerLM(spec), tokenizer, **kw)

    def with_frozen_reference(self) -> "NativePolicy":
        if self._has_adapter:
            return self
        ref = copy.deepcopy(self.model).eval()
        for p in ref.parameters():
            p.requires_grad = False
        self.reference_model = ref
        return self

    # protocol ------------------------------------------------------------
    @property
    def device(self) -> torch.device:
        return next(self.model.parameters()).device

    @property
    def vocab_size(self) -> int:
        return self.spec.vocab_size

    @property
    def has_adapter(self) -> bool:
        return self._has_adapter

    @property
    def max_length(self) -> int:
        return self.spec.block_size

    def trainable_parameters(self) -> List[nn.Parameter]:
        ps = [p for p in self.model.parameters() if p.requires_grad]
        if self.value_head is not None:
            ps += list(self.value_head.parameters())
        return ps

    @torch.no_grad()
    def generate(self, prompt_ids: torch.Tensor, settings: GenerationSettings) -> torch.Tensor:
        self.model.eval()
        prompt_ids = prompt_ids.to(self.device)
        out = generate_tokens(self.model, prompt_ids, settings.max_new_tokens, temperature=settings.temperature,
                              top_k=settings.top_k, top_p=settings.top_p, min_p=settings.min_p,
                              repetition_penalty=settings.repetition_penalty, use_cache=settings.use_cache,
                              stop_token_ids=settings.stop_token_ids)
        return out[:, prompt_ids.shape[1]:]

    def token_logits(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.model.full_logits(input_ids.to(self.device))

    def token_logprobs(self, input_ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Per-position ``log p(targets | input_ids)`` ``[B, T]`` (fused LM-head kernel on CUDA)."""
        return self.model.token_logprobs(input_ids.to(self.device), targets.to(self.device))

    def token_ce(self, input_ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Mean next-token CE over ``targets != -1`` through the fused LM-head kernel."""
        from rl_project_b200.ops.logprob import linear_cross_entropy

        h = self.model.forward_hidden(input_ids.to(self.device))
        return linear_cross_entropy(h.reshape(-1, h.shape[-1]), self.model.head_weight(),
                                    targets.to(self.device).reshape(-1))

    def _full(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor) -> torch.Tensor:
        full = torch.cat([prompt_ids.to(self.device), response_ids.to(self.device)], dim=1)
        if full.shape[1] > self.spec.block_size:
            raise ModelError(f"prompt+response length {full.shape[1]} exceeds block_size {self.spec.block_size}")
        return full

    def full_sequence_logits(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor) -> torch.Tensor:
        return self.model.full_logits(self._full(prompt_ids, response_ids))

    def _response_lp(self, h: torch.Tensor, full: torch.Tensor, q_len: int, with_entropy: bool = False):
        B, T, C = h.shape
        hs = h[:, q_len - 1: T - 1, :].reshape(-1, C)
        tg = full[:, q_len:].reshape(-1)
        lp, extra = linear_logprobs(hs, self.model.head_weight(), tg, with_entropy)
        R = T - q_len
        return lp.view(B, R), (extra.view(B, R) if with_entropy else None)

    def logprobs(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor,
                 response_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        full = self._full(prompt_ids, response_ids)
        h = self.model.forward_hidden(full)
        lp, _ = self._response_lp(h, full, prompt_ids.shape[1])
        if response_mask is not None:
            lp = lp * response_mask.to(lp.device, lp.dtype)
        return lp

    def logprobs_with_entropy(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor):
        full = self._full(prompt_ids, response_ids)
        h = self.model.forward_hidden(full)
        return self._response_lp(h, full, prompt_ids.shape[1], with_entropy=True)

    def values(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor) -> torch.Tensor:
        if self.value_head is None:
            raise ConfigError("values() requires value_head=True on the policy")
        h = self.model.forward_hidden(self._full(prompt_ids, response_ids))
        return self.value_head(h[:, -1, :].float()).float()

    def logprobs_and_values(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor):
        full = self._full(prompt_ids, response_ids)
        h = self.model.forward_hidden(full)
        lp, _ = self._response_lp(h, full, prompt_ids.shape[1])
        vals = self.value_head(h[:, -1, :].float()).float() if self.value_head is not None else None
        return lp, vals

    @contextmanager
    def reference(self) -> Iterator["NativePolicy"]:
        if self._has_adapter:
            set_lora_enabled(self.model, False)
            try:
                yield self
            finally:
                set_lora_enabled(self.model, True)
        elif self.reference_model is not None:
            live = self.model
            self.model = self.reference_model
            try:
                yield self
            finally:
                self.model = live
        else:
            raise ConfigError("no reference policy: call with_frozen_reference() or use an adapter",
                              hint="KL-regularised algorithms need a frozen reference.")

    # checkpoint ------------------------------------------------------------
    def state_for_checkpoint(self) -> Dict[str, Any]:
        st: Dict[str, Any] = {"model": self.model.state_dict()}
        if self._has_adapter:
            st["adapter"] = lora_state_dict(self.model)
        if self.value_head is not None:
            st["value_head"] = self.value_head.state_dict()
        return st

    def load_checkpoint_state(self, state: Mapping[str, Any]) -> None:
        from rl_project_b200.checkpoints.manager import load_model_state

        if "model" in state:
            load_model_state(self.model, state["model"], strict=False)
        if "adapter" in state and self._has_adapter:
            load_lora_state_dict(self.model, state["adapter"], strict=False)
        if "value_head" in state and self.value_head is not None:
            self.value_head.load_state_dict(state["value_head"])

    def encode(self, text: str) -> List[int]:
        return self.tokenizer.encode(text)

    def decode(self, ids) -> str:
        if isinstance(ids, torch.Tensor):
            ids = ids.tolist()
        return self.tokenizer.decode([int(t) for t in ids])

    def to(self, *args: Any, **kwargs: Any) -> "NativePolicy":  # type: ignore[override]
        super().to(*args, **kwargs)
        if self.reference_model is not None:
            self.reference_model.to(*args, **kwargs)
        return self



def has_lora_modules(model: nn.Module) -> bool:
    """True when ``model`` carries LoRA / QLoRA adapter layers (src/forgeline/models/policy.py:421-422)."""
    from rl_project_b200.models.adapters.lora import LoRALinear
    from rl_project_b200.models.adapters.qlora import QLoRALinear

    return any(isinstance(m, (LoRALinear, QLoRALinear)) for m in model.modules())
