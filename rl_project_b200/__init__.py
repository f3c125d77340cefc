"""rl_project_b200: a Blackwell-native (sm_100a) LLM post-training framework.

Framework layer in PyTorch (manifests, algorithms, trainer, checkpoints,
rollouts, serving); hot ops in hand-written CUDA for sm_100a loaded from the
in-tree extension ``rl_project_b200._C``; multi-GPU plumbing over
``torch.distributed`` (NCCL) plus NVLink peer-memory kernels.
"""

__version__ = "0.1.0"
