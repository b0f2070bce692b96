"""Tensor-parallel plan agreement: every TP peer must execute the same schedule.

A SHA-256 digest covers the forest (tree membership, node ranges), every
SegmentPlan (segments in insertion order, tokens, DFS events) and every PPO
ref; the 32-byte digest is all-gathered on the TP group as eight ``int64``
words *before* any model forward, and any mismatch raises on every peer.

Parity: verl/models/mcore/tpr/tp_validation.py:40-131.
"""

from __future__ import annotations

import hashlib
import json

import torch
import torch.distributed as dist


def _plan_bytes(h, plan, events=None) -> None:
    h.update(repr((plan.root_id, bool(plan.topology_only))).encode())
    for seg in plan.segments.values():
        terms = [(t.query_offset, t.target_token_id, float(t.weight), t.sample_id) for t in seg.loss_terms]
        h.update(json.dumps((seg.segment_id, seg.parent_id, seg.position_start, seg.prefix_length, seg.length, terms),
                            separators=(",", ":")).encode())
        h.update(seg.token_ids.numpy().tobytes())
    for ev in (plan.dfs_events() if events is None else events):
        h.update(f"{ev.kind.value}:{ev.segment_id};".encode())


def digest_segment_plan(plan, events=None) -> str:
    h = hashlib.sha256()
    _plan_bytes(h, plan, events)
    return h.hexdigest()


def digest_forest_plan(forest) -> str:
    h = hashlib.sha256()
    h.update(f"loss_tokens={forest.logical_loss_tokens};".encode())
    for ex in forest.trees:
        t = ex.tree
        h.update(json.dumps((t.uid, t.tree_index, list(t.member_rows), t.root_id), separators=(",", ":")).encode())
        for n in t.nodes.values():
            h.update(json.dumps((n.node_id, n.parent_id, n.segment.row, n.segment.start, n.segment.end,
                                 list(n.member_rows), list(n.terminal_rows), list(n.children)),
                                separators=(",", ":")).encode())
        _plan_bytes(h, ex.segment_plan)
        cols = getattr(ex.objective_refs, "columns", None)
        if cols is not None:
            h.update(cols.astype("<i8").tobytes())
        else:
            import numpy as np

            h.update(np.asarray([(r.segment_id, r.query_offset, r.target_token_id, r.sample_row, r.response_offset)
                                 for r in ex.objective_refs], dtype="<i8").reshape(-1, 5).tobytes())
    return h.hexdigest()


def assert_tp_plan_agreement(digest: str, *, tp_size: int, group=None, device=None) -> None:
    """All-gather the digest on the TP group; raise on every peer if any differs."""
    if tp_size == 1:
        return
    if tp_size < 1:
        raise ValueError("tp_size must be positive")
    if len(digest) != 64:
        raise ValueError("SHA256 digest must be a 64-character hex string")
    if not dist.is_available() or not dist.is_initialized():
        raise RuntimeError("TPR TP>1 requires an initialized distributed process group")
    if dist.get_world_size(group=group) != tp_size:
        raise RuntimeError("TPR TP group size differs from the engine TP config")
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    local = torch.tensor([int(digest[i:i + 8], 16) for i in range(0, 64, 8)], dtype=torch.int64, device=device)
    gathered = [torch.empty_like(local) for _ in range(tp_size)]
    dist.all_gather(gathered, local, group=group)
    if any(not torch.equal(g, local) for g in gathered):
        raise RuntimeError(f"TPR TP schedule mismatch on tp_rank={dist.get_rank(group=group)}: forest, SegmentPlan, "
                           "DFS events or PPO refs differ across model-parallel peers")
