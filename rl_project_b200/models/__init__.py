"""Model layer: transformer (GQA / MLA / NSA, MoE, MTP), adapters, quantisation, generation, policies, rewards."""

from rl_project_b200.models.loading import (build_model, load_model_from_checkpoint, load_policy_from_checkpoint,
                                            load_reward_model_from_checkpoint)
from rl_project_b200.models.policy import NativePolicy, ValueHead
from rl_project_b200.models.reward import EncoderRewardModel, SequenceRewardModel, bradley_terry_loss
from rl_project_b200.models.transformer.model import TransformerLM


def __getattr__(name):
    if name == "HFPolicy":
        from rl_project_b200.models.hf_policy import HFPolicy

        return HFPolicy
    raise AttributeError(name)
