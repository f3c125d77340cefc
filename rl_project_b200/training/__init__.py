"""Training: the shared Trainer plus every post-training algorithm."""

from rl_project_b200.training.common.trainer import PostTrainingAlgorithm, StepResult, Trainer
from rl_project_b200.training.dapo import DAPOAlgorithm, DAPOConfig
from rl_project_b200.training.distill import DistillationAlgorithm, DistillConfig
from rl_project_b200.training.dpo import DPOAlgorithm, DPOConfig
from rl_project_b200.training.grpo import GRPOAlgorithm, GRPOConfig
from rl_project_b200.training.ppo import PPOAlgorithm, PPOConfig
from rl_project_b200.training.pretrain import PretrainAlgorithm, PretrainConfig
from rl_project_b200.training.reward_model import RewardModelAlgorithm, RewardModelConfig
from rl_project_b200.training.rlvr import RLVRConfig, build_rlvr_algorithm
from rl_project_b200.training.sft import SFTAlgorithm, SFTConfig
