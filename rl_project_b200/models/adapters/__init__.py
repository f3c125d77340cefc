"""Parameter-efficient adapters: LoRA and QLoRA."""

from rl_project_b200.models.adapters.lora import (
    DEFAULT_TARGET_MODULES,
    LoRALinear,
    apply_lora,
    load_lora,
    load_lora_state_dict,
    lora_state_dict,
    merge_lora,
    save_lora,
    set_lora_enabled,
    trainable_parameter_report,
)
from rl_project_b200.models.adapters.qlora import QLoRALinear, apply_qlora
