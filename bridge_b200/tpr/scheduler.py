"""Fixed-topology scheduler and forest batch runner.

:class:`FixedTopologyScheduler` runs one validated Push/Pop stream against a
:class:`SegmentExecutor`.  The stream is first *lowered* to physical executions: a push that is
immediately followed by the pop of the same childless segment becomes one VISIT_LEAF (forward and
backward in one go, no prefix state kept); every other event stays a PUSH or a POP.  The scheduler
then executes that list, records the peak path length (prefix + segment tokens) and moves READY ->
RUNNING -> COMPLETED, or FAILED on any exception.

:class:`TPRBatchRunner` runs every tree of one mini-batch under one ``no_sync`` scope and finalises
gradients exactly once -- and not at all if any tree failed.

Parity: the public types and state machine of verl/models/mcore/tpr/fixed_topology_scheduler.py:32-210
and tpr_batch_runner.py:23-83; the lowering step and the code are this framework's own.
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
    """What one tree's schedule produced (traces, per-execution results, summed losses)."""

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
        """Segments that ran a forward: pushed ones plus directly visited leaves."""
        return len(self.forward_results) + len(self.direct_leaf_results)


def lower_events(plan: SegmentPlan, events: Sequence[SegmentEvent]) -> tuple[PhysicalExecution, ...]:
    """Physical executions of a validated event stream (adjacent push/pop of a leaf -> VISIT_LEAF)."""
    out: list[PhysicalExecution] = []
    it = iter(range(len(events)))
    for i in it:
        ev = events[i]
        nxt = events[i + 1] if i + 1 < len(events) else None
        if (ev.kind is SegmentEventKind.PUSH and nxt is not None and nxt.kind is SegmentEventKind.POP
                and nxt.segment_id == ev.segment_id and not plan.child_ids(ev.segment_id)):
            out.append(PhysicalExecution(PhysicalExecutionKind.VISIT_LEAF, ev.segment_id))
            next(it)                                 # the pop is part of the visit
        else:
            kind = PhysicalExecutionKind.PUSH if ev.kind is SegmentEventKind.PUSH else PhysicalExecutionKind.POP
            out.append(PhysicalExecution(kind, ev.segment_id))
    return tuple(out)


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
        for obj, cls in ((plan, SegmentPlan), (executor, SegmentExecutor)):
            if not isinstance(obj, cls):
                raise TypeError(f"expected a {cls.__name__}, got {type(obj).__name__}")
        problem = ("the executor was built for a different SegmentPlan object" if executor.plan is not plan else
                   "the executor has already failed" if executor.failed else
                   f"the executor still holds segments {list(executor.kv_stack.segment_ids)} on its KV stack"
                   if len(executor.kv_stack) else None)
        if problem:
            raise ValueError(f"cannot schedule tree {tree_index}: {problem}")
        self.events = plan.validate_events(plan.dfs_events() if events is None else events)
        self.executions = lower_events(plan, self.events)
        self.plan, self.executor = plan, executor
        self.event_profiler, self.tree_index = event_profiler, tree_index
        self.state = SchedulerState.READY

    def _execute(self, step: PhysicalExecution, out: dict) -> int:
        """Run one physical execution; return the path length it reached."""
        ex, sid = self.executor, step.segment_id
        if step.kind is PhysicalExecutionKind.VISIT_LEAF:
            r = ex.visit_leaf(sid)
            out["leaves"].append(r)
            out["losses"].append(r.backward)
            return r.forward.prefix_length + r.forward.suffix_length
        if step.kind is PhysicalExecutionKind.PUSH:
            out["fwd"].append(ex.push(sid))
            return ex.kv_stack.prefix_length
        r = ex.pop(sid)
        out["bwd"].append(r)
        out["losses"].append(r)
        return 0

    def run(self) -> TreeScheduleResult:
        if self.state is not SchedulerState.READY:
            raise RuntimeError(f"the scheduler of tree {self.tree_index} is {self.state.value}; it runs once, "
                               "from ready")
        self.state = SchedulerState.RUNNING
        out: dict[str, list] = {"fwd": [], "bwd": [], "leaves": [], "losses": []}
        peak = 0
        try:
            for i, step in enumerate(self.executions):
                stack = self.executor.kv_stack
                _mem_trace("EVENT_BEGIN", index=i, kind=step.kind.value, segment=step.segment_id,
                           path_tokens=stack.prefix_length, depth=len(stack))
                prof = None if self.event_profiler is None else self.event_profiler.begin(
                    self.plan.get(step.segment_id), kind=step.kind.value, tree_index=self.tree_index,
                    depth=self.plan.depth_of(step.segment_id))
                peak = max(peak, self._execute(step, out))
                if prof is not None:
                    self.event_profiler.end(prof)
                _mem_trace("EVENT_END", index=i, kind=step.kind.value, segment=step.segment_id)
            self.executor.kv_stack.assert_empty()
            losses = out["losses"]
            if not losses:
                raise RuntimeError(f"tree {self.tree_index}: the schedule ran no backward")
            loss_sum = torch.stack([r.loss_sum for r in losses]).sum()
            normalized = torch.stack([r.normalized_loss for r in losses]).sum()
            result = TreeScheduleResult(self.events, self.executions, tuple(out["fwd"]), tuple(out["bwd"]),
                                        tuple(out["leaves"]), loss_sum, normalized, peak)
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
