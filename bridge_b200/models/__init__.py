"""Policy models: Qwen3 dense, hybrid Gated-DeltaNet/attention, hybrid MoE."""

from .config import PRESETS, ModelConfig, get_config
from .decoder import DecoderModel, build_model
from .layers import DecoderLayer, RMSNorm, RotaryEmbedding, SwiGLUMLP, TPRGatedDeltaNet, TPRSelfAttention
