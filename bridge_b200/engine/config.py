"""Typed engine configuration with the reference's flag names.

Field names follow the verl/Megatron engine fields (``tpr_enabled``,
``tpr_cp_backend``, ``*_parallel_size``) and environment overrides keep the
reference's ``TPR_*`` variable names.

Parity: patches/3_5_megatron_engine.patch:9-10 (engine fields) and the env flags
read by verl/models/mcore/tpr/megatron_adapter.py:348-383.
"""

from __future__ import annotations

import os
from dataclasses import dataclass, field, replace


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    if v is None or v == "":
        return default
    try:
        return int(v)
    except ValueError as exc:
        raise ValueError(f"{name} must be an integer, got {v!r}") from exc


@dataclass(frozen=True)
class EngineConfig:
    tpr_enabled: bool = True
    tpr_cp_backend: str | None = None
    tensor_model_parallel_size: int = 1
    context_parallel_size: int = 1
    expert_model_parallel_size: int = 1
    pipeline_model_parallel_size: int = 1
    sequence_parallel: bool = False
    context_parallel_algo: str | None = None
    # execution
    executor: str = "forest"            # "forest" (batched levels) | "segment" (one segment per forward)
    forest_mode: str = "retain"         # "retain" (1F+1B per prefix) | "recompute" (2F+1B)
    token_budget: int = 8192            # max packed tokens per model forward
    tree_policy: str = "exact"
    turn_min_segment_tokens: int = 128
    log_prob_chunk_tokens: int = 0
    activation_offload: bool = False
    exec_profile: bool = False
    mem_trace: bool = False
    grad_comm_dtype: str = "bf16"
    # data-parallel gradient path: "auto" (NVLink P2P kernels + sharded optimizer on a single-node
    # CUDA group, NCCL otherwise), "nvlink" or "nccl"
    dp_comm: str = "auto"
    # sequence-parallel TP linears: "auto" (all-gather / reduce-scatter fused into the tcgen05 GEMM over
    # NVLink on a single-node CUDA group, NCCL otherwise), "nvlink" or "nccl"
    tp_comm: str = "auto"
    # ring / all-gather CP attention transport: "auto" (NVLink P2P gather + owner reduction on a
    # single-node CUDA group, NCCL otherwise), "nvlink" or "nccl"
    cp_comm: str = "auto"
    # MoE expert-parallel dispatch / combine: "auto" (NVLink P2P gathers on a single-node CUDA group,
    # NCCL all-to-all otherwise), "nvlink" or "nccl"
    ep_comm: str = "auto"
    # Gated DeltaNet under CP: "head" (head-parallel exchange, head-local state) or "sequence"
    # (sequence-sharded: per-piece affine state maps exchanged, no token activations moved)
    gdn_cp_mode: str = "head"
    extra: dict = field(default_factory=dict)

    def with_env(self) -> "EngineConfig":
        """Apply the ``TPR_*`` environment overrides."""
        kw = {}
        if "TPR_TREE_POLICY" in os.environ:
            kw["tree_policy"] = os.environ["TPR_TREE_POLICY"]
        if "TPR_TURN_MIN_SEGMENT_TOKENS" in os.environ:
            kw["turn_min_segment_tokens"] = _env_int("TPR_TURN_MIN_SEGMENT_TOKENS", 128)
        if "TPR_PPO_LOGPROB_CHUNK_TOKENS" in os.environ:
            kw["log_prob_chunk_tokens"] = _env_int("TPR_PPO_LOGPROB_CHUNK_TOKENS", 0)
        if os.environ.get("TPR_EXEC_PROFILE") == "1":
            kw["exec_profile"] = True
        if os.environ.get("TPR_MEM_TRACE") == "1":
            kw["mem_trace"] = True
        if "TPR_FOREST_MODE" in os.environ:
            kw["forest_mode"] = os.environ["TPR_FOREST_MODE"]
        if "TPR_TOKEN_BUDGET" in os.environ:
            kw["token_budget"] = _env_int("TPR_TOKEN_BUDGET", self.token_budget)
        if "TPR_EXECUTOR" in os.environ:
            kw["executor"] = os.environ["TPR_EXECUTOR"]
        if "TPR_EP_COMM" in os.environ:
            kw["ep_comm"] = os.environ["TPR_EP_COMM"]
        if "TPR_CP_COMM" in os.environ:
            kw["cp_comm"] = os.environ["TPR_CP_COMM"]
        if "TPR_TP_COMM" in os.environ:
            kw["tp_comm"] = os.environ["TPR_TP_COMM"]
        if "TPR_DP_COMM" in os.environ:
            kw["dp_comm"] = os.environ["TPR_DP_COMM"]
        if "TPR_ACTIVATION_OFFLOAD" in os.environ:
            kw["activation_offload"] = os.environ["TPR_ACTIVATION_OFFLOAD"] == "1"
        if "TPR_GDN_CP_MODE" in os.environ:
            kw["gdn_cp_mode"] = os.environ["TPR_GDN_CP_MODE"]
        cfg = replace(self, **kw) if kw else self
        if cfg.tree_policy not in ("exact", "qwen_turn"):
            raise ValueError(f"unknown TPR tree_policy: {cfg.tree_policy!r}")
        if cfg.ep_comm not in ("auto", "nvlink", "nccl"):
            raise ValueError(f"unknown ep_comm: {cfg.ep_comm!r}")
        if cfg.cp_comm not in ("auto", "nvlink", "nccl"):
            raise ValueError(f"unknown cp_comm: {cfg.cp_comm!r}")
        if cfg.tp_comm not in ("auto", "nvlink", "nccl"):
            raise ValueError(f"unknown tp_comm: {cfg.tp_comm!r}")
        if cfg.dp_comm not in ("auto", "nvlink", "nccl"):
            raise ValueError(f"unknown dp_comm: {cfg.dp_comm!r}")
        if cfg.gdn_cp_mode not in ("head", "sequence"):
            raise ValueError(f"unknown gdn_cp_mode: {cfg.gdn_cp_mode!r}")
        if cfg.log_prob_chunk_tokens < 0:
            raise ValueError("TPR_PPO_LOGPROB_CHUNK_TOKENS must be nonnegative")
        if cfg.turn_min_segment_tokens < 1:
            raise ValueError("TPR_TURN_MIN_SEGMENT_TOKENS must be a positive integer")
        return cfg
