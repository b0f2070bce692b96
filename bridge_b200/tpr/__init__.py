"""Tree-prefix-reuse core: planning, shards, prefix state, context and executors."""

from .context import (KVPair, SegmentBatchLayout, TPRAttentionBackend, TPRAttentionContext,
                      get_tpr_attention_context, use_tpr_attention_context)
from .dp_placement import DPPlacementPlan, plan_dta_dfs, plan_tpr_dta_dp, plan_verl_uid
from .forest_executor import ForestExecutor, ForestRunResult
from .kv_stack import KVStack, KVStackEntry, PastKVAnchors, PastKVSlice
from .prefix_state import (GDNLayerState, GDNPrefixAnchors, GDNPrefixState, KVPrefixAnchors, KVPrefixState,
                           PrefixState, PrefixStateEntry, PrefixStateStack, SegmentKV)
from .rope import build_sharded_rotary_pos_emb, build_suffix_rotary_pos_emb, sharded_position_ids
from .scheduler import (FixedTopologyScheduler, PhysicalExecution, PhysicalExecutionKind, SchedulerState,
                        TPRBatchResult, TPRBatchRunner, TreeScheduleResult)
from .segment_executor import (LeafVisitResult, SegmentBackwardResult, SegmentExecutor, SegmentForwardResult,
                               SegmentOutputs)
from .segment_plan import (PopSegment, PushSegment, SegmentEvent, SegmentEventKind, SegmentLossTerm, SegmentPlan,
                           SegmentSpec)
from .shard import (PaddedSequenceShard, PrefixShard, RangeSequenceShard, SequenceShard, iter_valid_sequence_slices,
                    make_hybrid_sequence_shard, make_ring_sequence_shard, maybe_pad_sequence_shard,
                    physical_sequence_shard, round_up_sequence_length)
from .tp_validation import assert_tp_plan_agreement, digest_forest_plan, digest_segment_plan
from .trajectory_tree import (SegmentRef, TrajectoryNode, TrajectoryTree, build_prompt_sibling_trees,
                              build_trajectory_trees)
from .trajectory_tree_turn import QWEN3_IM_END_TOKEN_ID, build_trajectory_trees_turn
from .tree_plan_builder import (ForestExecutionPlan, SegmentObjectiveRef, TreeExecutionPlan,
                                build_tree_execution_plans)
