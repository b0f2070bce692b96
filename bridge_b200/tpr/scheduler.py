"""Fixed-topology scheduler and forest batch runner.

:class:`FixedTopologyScheduler` executes one validated Push/Pop stream against
a :class:`SegmentExecutor`; an adjacent ``Push(x), Pop(x)`` of a leaf becomes a
single VISIT_LEAF.  It tracks the peak path length (prefix + segment tokens)
and moves READY -> RUNNING -> COMPLETED, or FAILED on any exception.

:class:`TPRBatchRunner` runs every tree of one mini-batch under one
``no_sync`` scope and finalises gradients exactly once -- and not at all if any
tree failed.

Parity: verl/models/mcore/tpr/fixed_topology_scheduler.py:32-210 and
verl/models/mcore/tpr/tpr_batch_runner.py:23-83.
"""

from __future__ import annotations

import os
from collections.abc import Callable, Sequence
from contextlib import nullcontext
from dataclasses import dataclass
from enum import Enum
from typing import Any

import torch
from torch import Tensor

from .segment_executor import LeafVisitResult, SegmentBackwardResult, SegmentExecutor, SegmentForwardResult
from .segment_plan import SegmentEvent, SegmentEventKind, SegmentPlan
from .tree_plan_builder import ForestExecutionPlan, TreeExecutionPlan


class SchedulerState(str, Enum):
    READY = "ready"
    RUNNING = "running"
    COMPLETED = "completed"
    FAILED = "failed"


class PhysicalExecutionKind(str, Enum):
    PUSH = "push"
    POP = "pop"
    VISIT_LEAF = "visit_leaf"


@dataclass(frozen=True, slots=True)
class PhysicalExecution:
    kind: PhysicalExecutionKind
    segment_id: int


@dataclass(frozen=True, slots=True)
class TreeScheduleResult:
    event_trace: tuple[SegmentEvent, ...]
    execution_trace: tuple[PhysicalExecution, ...]
    forward_results: tuple[SegmentForwardResult, ...]
    backward_results: tuple[SegmentBackwardResult, ...]
    direct_leaf_results: tuple[LeafVisitResult, ...]
    loss_sum: Tensor
    normalized_loss: Tensor
    peak_path_tokens: int

    @property
    def pushed_segment_count(self) -> int:
        return len(self.forward_results)

    @property
    def popped_segment_count(self) -> int:
        return len(self.backward_results)

    @property
    def direct_leaf_count(self) -> int:
        return len(self.direct_leaf_results)

    @property
    def executed_segment_count(self) -> int:
        return self.pushed_segment_count + self.direct_leaf_count


def _mem_trace(tag: str, **fields) -> None:
    if os.environ.get("TPR_MEM_TRACE", "0") != "1":
        return
    alloc = torch.cuda.memory_allocated() / 2**30 if torch.cuda.is_available() else 0.0
    resv = torch.cuda.memory_reserved() / 2**30 if torch.cuda.is_available() else 0.0
    body = " ".join(f"{k}={v}" for k, v in fields.items())
    print(f"TPR_MEM {tag} {body} alloc_gib={alloc:.3f} reserved_gib={resv:.3f}", flush=True)


class FixedTopologyScheduler:
    """Execute one immutable, validated DFS Push/Pop event stream."""

    def __init__(self, plan: SegmentPlan, executor: SegmentExecutor, *, events: Sequence[SegmentEvent] | None = None,
                 event_profiler=None, tree_index: int = 0) -> None:
        if not isinstance(plan, SegmentPlan):
            raise TypeError(f"plan must be SegmentPlan, got {type(plan).__name__}")
        if not isinstance(executor, SegmentExecutor):
            raise TypeError(f"executor must be SegmentExecutor, got {type(executor).__name__}")
        if executor.plan is not plan:
            raise ValueError("executor and scheduler must share the same SegmentPlan instance")
        if executor.failed:
            raise ValueError("executor is already failed")
        if len(executor.kv_stack):
            raise ValueError("executor KV stack must be empty before scheduling")
        self.events = plan.validate_events(tuple(plan.dfs_events()) if events is None else tuple(events))
        self.plan, self.executor = plan, executor
        self.event_profiler, self.tree_index = event_profiler, tree_index
        self.state = SchedulerState.READY

    def _leaf_pair(self, i: int) -> bool:
        if i + 1 >= len(self.events):
            return False
        a, b = self.events[i], self.events[i + 1]
        return (a.kind is SegmentEventKind.PUSH and b.kind is SegmentEventKind.POP and a.segment_id == b.segment_id
                and not self.plan.child_ids(a.segment_id))

    def run(self) -> TreeScheduleResult:
        if self.state is not SchedulerState.READY:
            raise RuntimeError(f"scheduler can only run from READY, current state is {self.state.value}")
        self.state = SchedulerState.RUNNING
        fwd, bwd, leaves, losses, trace = [], [], [], [], []
        peak = 0
        ex = self.executor
        try:
            i = 0
            while i < len(self.events):
                ev = self.events[i]
                leaf = self._leaf_pair(i)
                kind = "visit_leaf" if leaf else ev.kind.value
                _mem_trace("EVENT_BEGIN", index=i, kind=kind, segment=ev.segment_id,
                           path_tokens=ex.kv_stack.prefix_length, depth=len(ex.kv_stack))
                prof = None
                if self.event_profiler is not None:
                    prof = self.event_profiler.begin(self.plan.get(ev.segment_id), kind=kind,
                                                     tree_index=self.tree_index,
                                                     depth=self.plan.depth_of(ev.segment_id))
                if leaf:
                    r = ex.visit_leaf(ev.segment_id)
                    leaves.append(r)
                    losses.append(r.backward)
                    trace.append(PhysicalExecution(PhysicalExecutionKind.VISIT_LEAF, ev.segment_id))
                    peak = max(peak, r.forward.prefix_length + r.forward.suffix_length)
                    step = 2
                elif ev.kind is SegmentEventKind.PUSH:
                    fwd.append(ex.push(ev.segment_id))
                    trace.append(PhysicalExecution(PhysicalExecutionKind.PUSH, ev.segment_id))
                    peak = max(peak, ex.kv_stack.prefix_length)
                    step = 1
                else:
                    r = ex.pop(ev.segment_id)
                    bwd.append(r)
                    losses.append(r)
                    trace.append(PhysicalExecution(PhysicalExecutionKind.POP, ev.segment_id))
                    step = 1
                if prof is not None:
                    self.event_profiler.end(prof)
                _mem_trace("EVENT_END", index=i, kind=kind, segment=ev.segment_id)
                i += step
            ex.kv_stack.assert_empty()
            if not losses:
                raise RuntimeError("schedule produced no backward results")
            loss_sum = sum((r.loss_sum for r in losses[1:]), losses[0].loss_sum)
            normalized = sum((r.normalized_loss for r in losses[1:]), losses[0].normalized_loss)
            result = TreeScheduleResult(self.events, tuple(trace), tuple(fwd), tuple(bwd), tuple(leaves), loss_sum,
                                        normalized, peak)
        except Exception:
            self.state = SchedulerState.FAILED
            raise
        self.state = SchedulerState.COMPLETED
        return result


@dataclass(frozen=True, slots=True)
class TPRBatchResult:
    tree_results: tuple[Any, ...]
    normalized_loss: Tensor
    tree_count: int
    segment_count: int
    logical_loss_tokens: int


class TPRBatchRunner:
    """Run a whole mini-batch forest under one grad-sync scope; finalise once."""

    def __init__(self, *, run_tree: Callable[[TreeExecutionPlan], Any], finalize_gradients: Callable[[], None],
                 no_sync_context: Callable[[], Any] | None = None) -> None:
        if not callable(run_tree) or not callable(finalize_gradients):
            raise TypeError("run_tree and finalize_gradients must be callable")
        self.run_tree, self.finalize_gradients, self.no_sync_context = run_tree, finalize_gradients, no_sync_context
        self._ran = False

    def run(self, forest: ForestExecutionPlan) -> TPRBatchResult:
        if self._ran:
            raise RuntimeError("TPRBatchRunner is single-use for one optimizer mini-batch")
        self._ran = True
        if not isinstance(forest, ForestExecutionPlan) or not forest.trees:
            raise ValueError("forest must contain at least one executable tree")
        results, total = [], None
        with (nullcontext() if self.no_sync_context is None else self.no_sync_context()):
            for tree in forest.trees:
                out = self.run_tree(tree)
                loss = getattr(out, "normalized_loss", None)
                if not isinstance(loss, Tensor) or loss.numel() != 1:
                    raise TypeError("run_tree must return an object with scalar Tensor normalized_loss")
                results.append(out)
                total = loss.detach() if total is None else total + loss.detach()
        # Reached only when every tree succeeded: a failure above skips finalisation.
        self.finalize_gradients()
        return TPRBatchResult(tuple(results), total, len(forest.trees), forest.segment_count,
                              forest.logical_loss_tokens)
