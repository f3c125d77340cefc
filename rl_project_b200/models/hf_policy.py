"""HuggingFace causal LM (+ optional PEFT LoRA) behind the ``PolicyModel`` surface
(``src/forgeline/models/policy.py:225-418`` behaviour): left-padded tokenizer,
reference = ``disable_adapter()``, checkpoints keep only ``lora_`` tensors when
adapters are attached.  Optional: needs ``transformers`` (and ``peft`` for LoRA)."""

from __future__ import annotations

from contextlib import contextmanager
from typing import Any, Dict, Iterator, List, Mapping, Optional

import torch
import torch.nn as nn

from rl_project_b200.core.errors import ConfigError, OptionalDependencyError
from rl_project_b200.core.protocols import GenerationSettings
from rl_project_b200.models.policy import ValueHead
from rl_project_b200.ops.logprob import logprobs_from_logits


class _TokenizerAdapter:
    kind = "huggingface"

    def __init__(self, hf):
        self.hf = hf
        self.vocab_size = int(hf.vocab_size)

    def encode(self, text: str) -> List[int]:
        return self.hf.encode(text, add_special_tokens=False)

    def decode(self, ids) -> str:
        return self.hf.decode(list(ids), skip_special_tokens=True)

    def metadata(self) -> Dict[str, Any]:
        return {"tokenizer_type": "huggingface", "tokenizer_name": self.hf.name_or_path, "vocab_size": self.vocab_size}


class _HFSpec:
    def __init__(self, name: str, config: Any):
        self.name, self.config = name, config
        self.block_size = int(getattr(config, "max_position_embeddings", 4096))
        self.vocab_size = int(getattr(config, "vocab_size", 0))

    def to_dict(self) -> Dict[str, Any]:
        c = self.config
        return {"hf_model": self.name, "model_type": getattr(c, "model_type", ""), "vocab_size": self.vocab_size,
                "hidden_size": getattr(c, "hidden_size", None), "num_hidden_layers": getattr(c, "num_hidden_layers", None)}


class HFPolicy(nn.Module):
    backend = "huggingface"

    def __init__(self, model_name: str, *, lora_r: int = 8, lora_alpha: int = 16, lora_dropout: float = 0.05,
                 target_modules: Optional[List[str]] = None, load_in_8bit: bool = False, device_map: Any = "auto",
                 torch_dtype: Any = None, gradient_checkpointing: bool = True, value_head: bool = False,
                 use_lora: bool = True):
        super().__init__()
        try:
            from transformers import AutoModelForCausalLM, AutoTokenizer
        except ImportError as exc:
            raise OptionalDependencyError("transformers is not installed", hint="pip install transformers") from exc
        self.model_name = model_name
        self.hf_tokenizer = AutoTokenizer.from_pretrained(model_name, padding_side="left")
        if self.hf_tokenizer.pad_token is None:
            self.hf_tokenizer.pad_token = self.hf_tokenizer.eos_token
        kw: Dict[str, Any] = {"device_map": device_map}
        if torch_dtype is not None:
            kw["torch_dtype"] = torch_dtype
        if load_in_8bit:
            kw["load_in_8bit"] = True
        base = AutoModelForCausalLM.from_pretrained(model_name, **kw)
        self._has_adapter = False
        if use_lora:
            try:
                from peft import LoraConfig, TaskType, get_peft_model
            except ImportError as exc:
                raise OptionalDependencyError("peft is not installed", hint="pip install peft") from exc
            base = get_peft_model(base, LoraConfig(task_type=TaskType.CAUSAL_LM, r=lora_r, lora_alpha=lora_alpha,
                                                   lora_dropout=lora_dropout, bias="none",
                                                   target_modules=target_modules or ["q_proj", "k_proj", "v_proj",
                                                                                     "o_proj"]))
            self._has_adapter = True
        if gradient_checkpointing:
            if hasattr(base, "enable_input_require_grads"):
                base.enable_input_require_grads()
            base.gradient_checkpointing_enable()
        self.model = base
        self.reference_model = None  # set by with_frozen_reference() when no adapter provides the reference
        self.value_head: Optional[ValueHead] = (ValueHead(self.model.config.hidden_size).to(self.device)
                                                if value_head else None)
        self.pad_token_id = int(self.hf_tokenizer.pad_token_id)
        self.tokenizer = _TokenizerAdapter(self.hf_tokenizer)

    @property
    def device(self) -> torch.device:
        return next(self.model.parameters()).device

    @property
    def vocab_size(self) -> int:
        return int(self.model.config.vocab_size)

    @property
    def has_adapter(self) -> bool:
        return self._has_adapter

    @property
    def max_length(self) -> int:
        return int(getattr(self.model.config, "max_position_embeddings", 4096))

    @property
    def spec(self):
        return _HFSpec(self.model_name, self.model.config)

    def trainable_parameters(self) -> List[nn.Parameter]:
        ps = [p for p in self.model.parameters() if p.requires_grad]
        return ps + (list(self.value_head.parameters()) if self.value_head is not None else [])

    @torch.no_grad()
    def generate(self, prompt_ids: torch.Tensor, settings: GenerationSettings) -> torch.Tensor:
        self.model.eval()
        ids = prompt_ids.to(self.device)
        kw: Dict[str, Any] = dict(max_new_tokens=settings.max_new_tokens, pad_token_id=self.pad_token_id,
                                  eos_token_id=self.hf_tokenizer.eos_token_id, do_sample=settings.temperature > 0)
        if settings.temperature > 0:
            kw["temperature"] = settings.temperature
            if settings.top_p:
                kw["top_p"] = settings.top_p
            if settings.top_k:
                kw["top_k"] = settings.top_k
        out = self.model.generate(input_ids=ids, attention_mask=(ids != self.pad_token_id).long(), **kw)
        return out[:, ids.shape[1]:]

    def token_logits(self, input_ids: torch.Tensor) -> torch.Tensor:
        ids = input_ids.to(self.device)
        return self.model(input_ids=ids, attention_mask=(ids != self.pad_token_id).long()).logits

    def full_sequence_logits(self, prompt_ids, response_ids) -> torch.Tensor:
        return self.token_logits(torch.cat([prompt_ids.to(self.device), response_ids.to(self.device)], 1))

    def _forward(self, prompt_ids, response_ids, hidden: bool = False):
        full = torch.cat([prompt_ids.to(self.device), response_ids.to(self.device)], 1)
        return full, self.model(input_ids=full, attention_mask=(full != self.pad_token_id).long(),
                                output_hidden_states=hidden)

    def logprobs(self, prompt_ids, response_ids, response_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        full, out = self._forward(prompt_ids, response_ids)
        lp = logprobs_from_logits(out.logits[:, :-1], full[:, 1:])[:, prompt_ids.shape[1] - 1:]
        return lp * response_mask.to(lp.device, lp.dtype) if response_mask is not None else lp

    def token_logprobs(self, input_ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Per-position ``log p(targets | input_ids)`` ``[B, T]``; 0 where ``targets == -1``."""
        logits = self.token_logits(input_ids).float()
        tg = targets.to(logits.device)
        lp = torch.log_softmax(logits, -1).gather(-1, tg.clamp(min=0)[..., None])[..., 0]
        return lp * (tg >= 0)

    def token_ce(self, input_ids: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """Mean next-token cross-entropy over ``targets != -1`` (the SFT / pretrain loss)."""
        logits = self.token_logits(input_ids)
        return nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]),
                                           targets.to(logits.device).reshape(-1), ignore_index=-1)

    def logprobs_with_entropy(self, prompt_ids, response_ids):
        """Response-token log-probs and the policy's entropy at each response position."""
        full, out = self._forward(prompt_ids, response_ids)
        logits = out.logits[:, prompt_ids.shape[1] - 1:-1].float()
        logp = torch.log_softmax(logits, -1)
        lp = logp.gather(-1, full[:, prompt_ids.shape[1]:, None])[..., 0]
        ent = -(logp.exp() * logp).sum(-1)
        return lp, ent

    def with_frozen_reference(self) -> "HFPolicy":
        """A frozen copy of the initial weights as the KL reference when no adapter is attached (with LoRA the
        reference is the base model with the adapter disabled)."""
        if self._has_adapter:
            return self
        import copy

        ref = copy.deepcopy(self.model).eval()
        for p in ref.parameters():
            p.requires_grad = False
        self.reference_model = ref
        return self

    def values(self, prompt_ids, response_ids) -> torch.Tensor:
        if self.value_head is None:
            raise ConfigError("values() requires value_head=True on the policy")
        _, out = self._forward(prompt_ids, response_ids, hidden=True)
        return self.value_head(out.hidden_states[-1][:, -1].float())

    def logprobs_and_values(self, prompt_ids, response_ids):
        full, out = self._forward(prompt_ids, response_ids, hidden=self.value_head is not None)
        lp = logprobs_from_logits(out.logits[:, :-1], full[:, 1:])[:, prompt_ids.shape[1] - 1:]
        v = self.value_head(out.hidden_states[-1][:, -1].float()) if self.value_head is not None else None
        return lp, v

    @contextmanager
    def reference(self) -> Iterator["HFPolicy"]:
        if self._has_adapter:
            with self.model.disable_adapter():
                yield self
            return
        ref = getattr(self, "reference_model", None)
        if ref is None:
            raise ConfigError("HFPolicy reference needs LoRA adapters (use_lora=True) or with_frozen_reference()")
        live = self.model
        self.model = ref
        try:
            yield self
        finally:
            self.model = live

    def state_for_checkpoint(self) -> Dict[str, Any]:
        st: Dict[str, Any] = {}
        if self._has_adapter:
            st["adapter"] = {k: v.detach().cpu() for k, v in self.model.state_dict().items() if "lora_" in k}
        else:
            st["model"] = self.model.state_dict()
        if self.value_head is not None:
            st["value_head"] = self.value_head.state_dict()
        return st

    def load_checkpoint_state(self, state: Mapping[str, Any]) -> None:
        for key in ("adapter", "model"):
            if key in state:
                self.model.load_state_dict(dict(state[key]), strict=False)
        if "value_head" in state and self.value_head is not None:
            self.value_head.load_state_dict(state["value_head"])

    def save_adapter(self, path: str) -> None:
        self.model.save_pretrained(path)
        self.hf_tokenizer.save_pretrained(path)
        if self.value_head is not None:
            torch.save(self.value_head.state_dict(), f"{path}/value_head.pt")

    def encode(self, text: str) -> List[int]:
        return self.tokenizer.encode(text)

    def decode(self, ids) -> str:
        return self.tokenizer.decode(ids.tolist() if isinstance(ids, torch.Tensor) else ids)
