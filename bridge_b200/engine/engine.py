"""Training engine: model + FP32-master AdamW + parallel groups + TPR entry points.

``TPREngine.forward_backward_batch(data, loss_function)`` is the call a PPO
trainer makes once per mini-batch (it dispatches to
:func:`run_tpr_forward_backward_batch` when ``tpr_enabled``), followed by
``optimizer_step()``.  ``train_step`` does both.

Parity: the verl ``MegatronEngine`` integration of
patches/3_5_megatron_engine.patch:1-55 (tpr_enabled / tpr_cp_backend fields,
module-spec install before model construction, PPO dispatch after
batch_num_tokens/dp_size are attached and before micro-batching).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from torch import nn

from ..models.config import ModelConfig
from ..models.decoder import DecoderModel, build_model
from ..parallel.dp import DataParallelGradReducer
from ..parallel.groups import ParallelState, build_parallel_state
from .config import EngineConfig
from .optim import AdamWConfig, MixedPrecisionAdamW


def _use_nvlink_dp(mode: str, device: torch.device, group) -> bool:
    """The fused NVLink data-parallel path needs CUDA, a single-node group of 2..8 ranks."""
    import os

    import torch.distributed as dist

    if mode == "nccl" or device.type != "cuda" or group is None:
        return False
    n = dist.get_world_size(group)
    local = int(os.environ.get("LOCAL_WORLD_SIZE", dist.get_world_size()))
    ok = 1 < n <= 8 and local >= dist.get_world_size()
    if mode == "nvlink" and not ok:
        raise ValueError("dp_comm='nvlink' needs a single-node data-parallel group of 2..8 GPUs")
    return ok


class TPREngine:
    def __init__(self, model_config: ModelConfig, engine_config: EngineConfig = EngineConfig(),
                 optim_config: AdamWConfig = AdamWConfig(), *, device=None, seed: int = 0,
                 parallel_state: ParallelState | None = None, model: nn.Module | None = None) -> None:
        self.model_config = model_config
        self.engine_config = engine_config.with_env()
        ec = self.engine_config
        if ec.pipeline_model_parallel_size != 1:
            raise NotImplementedError("TPR does not support pipeline parallelism")
        self.parallel = parallel_state or build_parallel_state(ec.tensor_model_parallel_size,
                                                               ec.context_parallel_size,
                                                               ec.expert_model_parallel_size)
        from ..parallel.cp_p2p import set_cp_comm_mode
        from ..parallel.ep_p2p import set_ep_comm_mode
        from ..parallel.gdn_state import set_gdn_cp_mode
        from ..parallel.tp_fused import set_tp_comm_mode

        set_tp_comm_mode(ec.tp_comm)
        set_cp_comm_mode(ec.cp_comm)
        set_ep_comm_mode(ec.ep_comm)
        set_gdn_cp_mode(ec.gdn_cp_mode)
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device)
        if model is None:
            from .api import install_tpr_module_spec

            provider = install_tpr_module_spec(lambda: build_model(
                model_config, device=self.device, seed=seed, tp_group=self.parallel.tp_group,
                sequence_parallel=ec.sequence_parallel, ep_group=self.parallel.ep_group))
            model = provider()
        self.module = [model]
        grad_group = self.parallel.dp_cp_group if (self.parallel.dp * self.parallel.cp) > 1 else None
        if self.parallel.tp == 1 and grad_group is None and self.parallel.dp > 1:
            grad_group = self.parallel.dp_group
        comm = torch.bfloat16 if ec.grad_comm_dtype == "bf16" else torch.float32
        self.symm_heap = None
        if _use_nvlink_dp(ec.dp_comm, self.device, grad_group):
            from ..parallel.symmetric import SymmetricHeap
            from .optim import ShardedNVLinkAdamW

            self.symm_heap = SymmetricHeap(grad_group, self.device)
            self.optimizer = ShardedNVLinkAdamW(model, optim_config, self.symm_heap,
                                                tp_group=self.parallel.tp_group if self.parallel.tp > 1 else None)
            self.grad_reducer = DataParallelGradReducer(None)   # reduction happens inside optimizer.step()
        else:
            self.optimizer = MixedPrecisionAdamW(model, optim_config)
            self.grad_reducer = DataParallelGradReducer(grad_group, comm_dtype=comm)
        self.enable_routing_replay = False
        self.last_metrics: dict[str, Any] = {}

    # -- verl engine surface -------------------------------------------------------
    @property
    def model(self) -> DecoderModel:
        return self.module[0]

    def get_data_parallel_size(self) -> int:
        return self.parallel.dp

    def get_data_parallel_group(self):
        return self.parallel.dp_group

    def finalize_model_grads(self) -> None:
        """TP sum of replicated-but-partial gradients (qk-norm / GDN norm weights, norms under SP), then
        the data-parallel reduction."""
        tp = self.parallel.tp_group
        if tp is not None and self.parallel.tp > 1 and not getattr(self.optimizer, "handles_tp_partial_grads", False):
            import torch.distributed as dist

            for p in self.model.parameters():
                if getattr(p, "tp_partial_grad", False):
                    dist.all_reduce(p.main_grad, group=tp)
        self.grad_reducer.finalize(self.optimizer.grad_buffers())

    def zero_grad(self) -> None:
        self.optimizer.zero_grad()

    def forward_backward_batch(self, data: Any, loss_function=None, *, forward_only: bool = False) -> dict:
        from .api import TPR_REQUEST_KEY, run_tpr_forward_backward, run_tpr_forward_backward_batch

        if not self.engine_config.tpr_enabled:
            raise RuntimeError("this engine runs TPR schedules only; set tpr_enabled=True")
        if isinstance(data, dict) and TPR_REQUEST_KEY in data:
            return run_tpr_forward_backward(self, data[TPR_REQUEST_KEY])
        return run_tpr_forward_backward_batch(self, data, loss_function, forward_only=forward_only)

    def optimizer_step(self) -> torch.Tensor:
        norm = self.optimizer.step()
        self.optimizer.zero_grad()
        return norm

    def train_step(self, data: Any, loss_function=None) -> dict:
        out = self.forward_backward_batch(data, loss_function)
        out["grad_norm"] = self.optimizer_step()
        if self.symm_heap is not None:
            self.symm_heap.check()
        return out
