"""Opt-in execution profiling for TPR schedules (``TPR_EXEC_PROFILE=1``).

:class:`SegmentEventProfiler` brackets every Push / Pop / VisitLeaf event (segment executor) or
push-chunk / visit-chunk / pop-chunk phase (forest executor) with a pair of CUDA events on the
current stream, an NVTX range (visible to ncu / nsys), and allocator peak snapshots.  Nothing
synchronises per event; :meth:`materialize` is called once after the mini-batch's final
synchronize.  Peaks are reset per event (``reset_peak_memory_stats``) so each record carries the
event's own peak; the overall maximum is the max over records.

:func:`max_over_ranks` turns per-rank device times into the rank-max critical path (the timing
convention for every multi-GPU number).

Parity: verl/models/mcore/tpr/segment_event_profiler.py:15-76 (per-event device events + allocator
peaks without per-event synchronisation) and the TPR_MEM_TRACE / stage timings of
megatron_adapter.py:348-366.
"""

from __future__ import annotations

import time
from typing import Any

import torch
import torch.distributed as dist


class SegmentEventProfiler:
    def __init__(self, *, nvtx: bool = True) -> None:
        self._pending: list[dict[str, Any]] = []
        self.nvtx = nvtx and torch.cuda.is_available()
        self.max_allocated_bytes = 0
        self.max_reserved_bytes = 0

    def _cuda(self) -> bool:
        return torch.cuda.is_available()

    def begin(self, segment=None, *, kind: str, tree_index: int = 0, depth: int = 0, tokens: int | None = None,
              label: str | None = None) -> dict:
        rec: dict[str, Any] = {"kind": kind, "tree_index": int(tree_index), "depth": int(depth),
                               "cpu_start": time.perf_counter()}
        if segment is not None:
            rec.update(segment_id=int(segment.segment_id), parent_id=segment.parent_id, length=int(segment.length),
                       prefix_length=int(segment.prefix_length))
        if tokens is not None:
            rec["tokens"] = int(tokens)
        if self._cuda():
            self.max_allocated_bytes = max(self.max_allocated_bytes, torch.cuda.max_memory_allocated())
            self.max_reserved_bytes = max(self.max_reserved_bytes, torch.cuda.max_memory_reserved())
            torch.cuda.reset_peak_memory_stats()
            rec["alloc_before_bytes"] = torch.cuda.memory_allocated()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            rec["_start"], rec["_end"] = start, end
            if self.nvtx:
                torch.cuda.nvtx.range_push(label or f"tpr/{kind}")
        return rec

    def end(self, rec: dict) -> None:
        rec["cpu_enqueue_ms"] = (time.perf_counter() - rec.pop("cpu_start")) * 1e3
        if self._cuda():
            rec["_end"].record()
            if self.nvtx:
                torch.cuda.nvtx.range_pop()
            rec["alloc_after_bytes"] = torch.cuda.memory_allocated()
            rec["peak_allocated_bytes"] = torch.cuda.max_memory_allocated()
            rec["peak_reserved_bytes"] = torch.cuda.max_memory_reserved()
            self.max_allocated_bytes = max(self.max_allocated_bytes, rec["peak_allocated_bytes"])
            self.max_reserved_bytes = max(self.max_reserved_bytes, rec["peak_reserved_bytes"])
        self._pending.append(rec)

    def materialize(self) -> list[dict]:
        """Per-event records with ``device_ms``; call once after the final synchronize."""
        out = []
        for rec in self._pending:
            r = {k: v for k, v in rec.items() if not k.startswith("_")}
            if "_start" in rec:
                r["device_ms"] = float(rec["_start"].elapsed_time(rec["_end"]))
            out.append(r)
        return out

    def summary(self) -> dict:
        recs = self.materialize()
        by_kind: dict[str, float] = {}
        for r in recs:
            by_kind[r["kind"]] = by_kind.get(r["kind"], 0.0) + r.get("device_ms", 0.0)
        return {"events": len(recs), "device_ms_by_kind": by_kind, "max_allocated_bytes": self.max_allocated_bytes,
                "max_reserved_bytes": self.max_reserved_bytes}


class _Null:
    def begin(self, *a, **k):
        return None

    def end(self, rec) -> None:
        pass


NULL_PROFILER = _Null()


def max_over_ranks(value: float, group=None, device=None) -> float:
    """Max of a per-rank scalar over the group (identity without an initialised process group)."""
    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    dev = device or (torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu")
    t = torch.tensor([float(value)], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
