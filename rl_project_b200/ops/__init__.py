"""Hot ops of the framework, each backed by a hand-written sm_100a kernel on CUDA.

``rms_norm``/``add_rms_norm`` (csrc/norm.cu), ``rope_split_qkv`` (csrc/rope.cu),
``swiglu``/``gelu_tanh`` (csrc/swiglu.cu), ``linear_logprobs``/
``linear_cross_entropy`` (csrc/logprob.cu), ``embedding`` (csrc/embedding.cu),
``FusedAdamW`` (csrc/adamw.cu), attention (ops/attention.py).
"""

from rl_project_b200.ops._ext import available as native_available
from rl_project_b200.ops.activation import gelu_tanh, swiglu
from rl_project_b200.ops.attention import attention_reference, causal_attention
from rl_project_b200.ops.embedding import embedding
from rl_project_b200.ops.linear import linear, matmul_nt
from rl_project_b200.ops.logprob import linear_cross_entropy, linear_logprobs, logprobs_from_logits
from rl_project_b200.ops.norm import add_rms_norm, rms_norm
from rl_project_b200.ops.rope import RopeTable, apply_rope, rope_inv_freq, rope_split_qkv
