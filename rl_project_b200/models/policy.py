"""Policies over the native transformer (the ``PolicyModel`` protocol; capabilities of
``src/forgeline/models/policy.py:31-222``).

``NativePolicy`` is organised around one scoring pass.  ``_score(prompt, response, wants)`` runs the trunk
once over ``[prompt | response]`` and evaluates only the heads a caller asks for on its hidden states:
``"logprobs"`` (per-response-token log-probs through the fused LM-head log-softmax kernel, no ``[B, T, V]``
tensor), ``"entropy"`` (from the same kernel pass) and ``"value"`` (the value head on the last position).
Every public scoring method (``logprobs``, ``logprobs_with_entropy``, ``values``, ``logprobs_and_values``)
is a selection over it, so a PPO step that needs log-probs and values pays one forward.

The frozen reference is either the live model with its adapters switched off (LoRA / QLoRA: no second copy
of the weights) or a detached frozen copy; ``reference()`` swaps it in for the duration of a ``with`` block.
Checkpoint dicts are ``{model, adapter, value_head}`` (the reference's keys); ``_PARTS`` lists how each part
is saved and restored.
"""

from __future__ import annotations

import copy
from contextlib import contextmanager
from typing import Any, Callable, Dict, FrozenSet, Iterator, List, Mapping, Optional, Tuple

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
    """Scalar value from a hidden state: dropout, a half-width GELU layer, a linear read-out (parameter names
    ``net.1`` / ``net.3`` are the checkpoint format)."""

    def __init__(self, hidden_size: int, dropout: float = 0.1):
        super().__init__()
        self.net = nn.Sequential(nn.Dropout(dropout), nn.Linear(hidden_size, hidden_size // 2), nn.GELU(),
                                 nn.Linear(hidden_size // 2, 1))

    def forward(self, hidden: torch.Tensor) -> torch.Tensor:
        first = self.net[1]
        return self.net(hidden.to(first.weight.dtype))[..., 0]


def token_logprobs_from_logits(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    return logprobs_from_logits(logits, labels)


# adapter method -> function that injects it into a model
_ADAPTERS: Dict[str, Callable[..., nn.Module]] = {"lora": apply_lora, "qlora": apply_qlora}


class NativePolicy(nn.Module):
    backend = "native"

    def __init__(self, model: TransformerLM, tokenizer: Any, *, pad_token_id: int = 0,
                 adapter: Optional[AdapterConfig] = None, reference_model: Optional[TransformerLM] = None,
                 value_head: bool = False):
        super().__init__()
        self.model, self.tokenizer, self.pad_token_id = model, tokenizer, pad_token_id
        self.spec: ModelSpec = model.spec
        self.adapter = adapter or AdapterConfig()
        inject = _ADAPTERS.get(self.adapter.method)
        if inject is not None:
            a = self.adapter
            inject(model, a.rank, a.alpha, a.dropout, a.target_modules or None)
        self._has_adapter = inject is not None
        self.reference_model = reference_model
        self.value_head: Optional[ValueHead] = ValueHead(self.spec.n_embd) if value_head else None

    @classmethod
    def from_spec(cls, spec: ModelSpec, tokenizer: Any, **kw: Any) -> "NativePolicy":
        return cls(TransformerLM(spec), tokenizer, **kw)

    def with_frozen_reference(self) -> "NativePolicy":
        """Keep a frozen copy of the current weights as the reference (adapter policies need none: the
        reference is the model with its adapters off)."""
        if not self._has_adapter:
            self.reference_model = copy.deepcopy(self.model).eval().requires_grad_(False)
        return self

    # ------------------------------------------------------------ protocol properties
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
        head = list(self.value_head.parameters()) if self.value_head is not None else []
        return [p for p in self.model.parameters() if p.requires_grad] + head

    # ------------------------------------------------------------ generation
    @torch.no_grad()
    def generate(self, prompt_ids: torch.Tensor, settings: GenerationSettings) -> torch.Tensor:
        """Sampled continuation tokens only (the prompt is not repeated)."""
        self.model.eval()
        prompt_ids = prompt_ids.to(self.device)
        s = settings
        out = generate_tokens(self.model, prompt_ids, s.max_new_tokens, temperature=s.temperature, top_k=s.top_k,
                              top_p=s.top_p, min_p=s.min_p, repetition_penalty=s.repetition_penalty,
                              use_cache=s.use_cache, stop_token_ids=s.stop_token_ids)
        return out[:, prompt_ids.shape[1]:]

    # ------------------------------------------------------------ whole-sequence scoring
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

    # ------------------------------------------------------------ prompt / response scoring
    def _joined(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor) -> torch.Tensor:
        dev = self.device
        full = torch.cat([prompt_ids.to(dev), response_ids.to(dev)], dim=1)
        if full.shape[1] > self.spec.block_size:
            raise ModelError(f"prompt+response length {full.shape[1]} exceeds block_size {self.spec.block_size}")
        return full

    def _score(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor,
               wants: FrozenSet[str]) -> Dict[str, torch.Tensor]:
        full = self._joined(prompt_ids, response_ids)
        h = self.model.forward_hidden(full)
        out: Dict[str, torch.Tensor] = {}
        if wants & {"logprobs", "entropy"}:
            # position t predicts token t + 1: the response tokens are predicted from positions q - 1 .. T - 2
            B, T, C = h.shape
            q = prompt_ids.shape[1]
            lp, ent = linear_logprobs(h[:, q - 1:T - 1].reshape(-1, C), self.model.head_weight(),
                                      full[:, q:].reshape(-1), "entropy" in wants)
            out["logprobs"] = lp.view(B, T - q)
            if "entropy" in wants:
                out["entropy"] = ent.view(B, T - q)
        if "value" in wants:
            if self.value_head is None:
                raise ConfigError("values() requires value_head=True on the policy")
            out["value"] = self.value_head(h[:, -1].float()).float()
        return out

    def logprobs(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor,
                 response_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        lp = self._score(prompt_ids, response_ids, frozenset({"logprobs"}))["logprobs"]
        return lp if response_mask is None else lp * response_mask.to(lp.device, lp.dtype)

    def logprobs_with_entropy(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor):
        r = self._score(prompt_ids, response_ids, frozenset({"logprobs", "entropy"}))
        return r["logprobs"], r["entropy"]

    def values(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor) -> torch.Tensor:
        return self._score(prompt_ids, response_ids, frozenset({"value"}))["value"]

    def logprobs_and_values(self, prompt_ids: torch.Tensor, response_ids: torch.Tensor):
        wants = frozenset({"logprobs", "value"} if self.value_head is not None else {"logprobs"})
        r = self._score(prompt_ids, response_ids, wants)
        return r["logprobs"], r.get("value")

    # ------------------------------------------------------------ frozen reference
    @contextmanager
    def reference(self) -> Iterator["NativePolicy"]:
        """Score with the reference policy inside the block: adapters off, or the frozen copy swapped in."""
        if self._has_adapter:
            set_lora_enabled(self.model, False)
            try:
                yield self
            finally:
                set_lora_enabled(self.model, True)
            return
        if self.reference_model is None:
            raise ConfigError("no reference policy: call with_frozen_reference() or use an adapter",
                              hint="KL-regularised algorithms need a frozen reference.")
        live, self.model = self.model, self.reference_model
        try:
            yield self
        finally:
            self.model = live

    # ------------------------------------------------------------ checkpoint
    def _parts(self) -> List[Tuple[str, Callable[[], Any], Callable[[Any], None]]]:
        """(key, save, restore) of every part this policy carries."""
        from rl_project_b200.checkpoints.manager import load_model_state

        parts = [("model", self.model.state_dict, lambda st: load_model_state(self.model, st, strict=False))]
        if self._has_adapter:
            parts.append(("adapter", lambda: lora_state_dict(self.model),
                          lambda st: load_lora_state_dict(self.model, st, strict=False)))
        if self.value_head is not None:
            parts.append(("value_head", self.value_head.state_dict, self.value_head.load_state_dict))
        return parts

    def state_for_checkpoint(self) -> Dict[str, Any]:
        return {key: save() for key, save, _ in self._parts()}

    def load_checkpoint_state(self, state: Mapping[str, Any]) -> None:
        for key, _, restore in self._parts():
            if key in state:
                restore(state[key])

    # ------------------------------------------------------------ text
    def encode(self, text: str) -> List[int]:
        return self.tokenizer.encode(text)

    def decode(self, ids) -> str:
        seq = ids.tolist() if isinstance(ids, torch.Tensor) else ids
        return self.tokenizer.decode([int(t) for t in seq])

    def to(self, *args: Any, **kwargs: Any) -> "NativePolicy":  # type: ignore[override]
        super().to(*args, **kwargs)
        if self.reference_model is not None:
            self.reference_model.to(*args, **kwargs)
        return self


def has_lora_modules(model: nn.Module) -> bool:
    """True when ``model`` carries LoRA / QLoRA adapter layers (src/forgeline/models/policy.py:421-422)."""
    from rl_project_b200.models.adapters.lora import LowRankAdapter

    return any(isinstance(m, LowRankAdapter) for m in model.modules())
