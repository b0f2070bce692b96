"""Hot ops: sm_100a CUDA kernels on CUDA tensors, PyTorch formulations on CPU."""

from .activation import swiglu
from .attention import rectangular_causal_attention, tree_attention
from .gdn import causal_conv1d, chunk_gated_delta_rule
from .logprob import fused_lm_head_logprob
from .norm import qk_norm_rope, rmsnorm
from .ppo import PPOLossConfig, ppo_loss
