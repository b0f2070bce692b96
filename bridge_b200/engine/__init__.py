"""Training engine and public TPR entry points."""

from .api import (TPR_REQUEST_KEY, TPRForwardBackwardRequest, install_tpr_module_spec, make_tpr_module_spec_provider,
                  replace_self_attention_with_tpr, run_tpr_forward_backward, run_tpr_forward_backward_batch)
from .config import EngineConfig
from .engine import TPREngine
from .optim import AdamWConfig, MixedPrecisionAdamW
