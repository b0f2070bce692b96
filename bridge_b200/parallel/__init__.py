"""Parallelism: TP layers, CP backends (all-gather, Ulysses, ring, hybrid), GDN CP, DP, groups."""

from .backend import (ALLGATHER_CP_BACKEND, HYBRID_CP_BACKEND, MINDSPEED_ALLGATHER_CP_ALGO,
                      MINDSPEED_HYBRID_CP_ALGO, MINDSPEED_RING_CP_ALGO, MINDSPEED_ULYSSES_CP_ALGO, RING_CP_BACKEND,
                      ULYSSES_CP_BACKEND, AllGatherCPBackend, HybridCPBackend, RingCPBackend, TPRCPBackend,
                      UlyssesCPBackend, resolve_tpr_cp_backend)
from .execution_context import (HybridLocalKVBlock, LocalKVBlock, RingLocalKVBlock, ShardedPastKVAnchors,
                                accumulate_sharded_past_anchor_gradients, build_sharded_past_anchors,
                                resolve_cp_group)
from .allgather_attention import AllGatherCPAttentionBackend, all_gather_sequence, allgather_cp_rectangular_attention
from .ulysses_attention import (UlyssesCPAttentionBackend, head_to_sequence, sequence_to_head,
                                ulysses_cp_rectangular_attention)
from .ring_attention import (RingBlockKind, RingCPAttentionBackend, classify_ring_block, merge_attention,
                             ordinary_ring_cp_attention, ring_cp_attention)
from .hybrid_attention import (HybridCPAttentionBackend, HybridCPTopology, hybrid_cp_rectangular_attention,
                               resolve_mindspeed_hybrid_topology)
from .engine_runtime import TPREngineCPRuntime, aggregate_cp_loss, resolve_engine_cp_runtime
from .groups import ParallelState, build_parallel_state, collective_probe, init_distributed
from .gdn_state import forward_gdn_cp_with_state, gdn_cp_state_shapes
from .gdn_tree import GDNCPBranchExecutor, GDNCPStack
