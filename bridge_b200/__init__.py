"""bridge_b200: tree-prefix-reuse RL policy training, written for NVIDIA B200 (sm_100a).

The public surface mirrors the verl TPR extension (``verl.models.mcore.tpr``):
planning (tries, plans, events), prefix state, the Push/Pop executor and
scheduler, CP backends, the PPO objective and the engine entry points.
"""

from .engine import (TPR_REQUEST_KEY, EngineConfig, TPREngine, TPRForwardBackwardRequest, install_tpr_module_spec,
                     make_tpr_module_spec_provider, replace_self_attention_with_tpr, run_tpr_forward_backward,
                     run_tpr_forward_backward_batch)
from .models import ModelConfig, TPRGatedDeltaNet, TPRSelfAttention, build_model, get_config
from .ops import rectangular_causal_attention
from .parallel import *  # noqa: F401,F403
from .rl import SegmentPPOObjectiveAdapter
from .tpr import *  # noqa: F401,F403

__version__ = "0.1.0"
