"""PPO objective over the deduplicated token tree.

Each supervised logical token (one :class:`SegmentObjectiveRef`) is predicted
by a *physical* query row of a segment.  Refs that share ``(query row, target,
temperature)`` -- duplicate trajectories -- share one log-prob computation but
keep separate loss terms, so the loss equals the flattened batch exactly.

All per-ref PPO inputs (old log-prob, advantage, optional importance weight)
are flattened once per mini-batch on the host and copied to the device in one
transfer; a segment (or a packed chunk of segments) then only gathers rows.
The loss uses verl's global ``batch_num_tokens / dp_size`` normaliser, so the
per-segment losses add up to the mini-batch objective with no per-tree
division.

Parity: verl/models/mcore/tpr/objective_adapter.py:53-373
(SegmentPPOObjectiveAdapter.bind_tree / compute_loss, dedupe on
(query, target, temperature), vanilla + token-mean only).
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch
from torch import Tensor

from ..ops._ext import on_gpu
from ..ops.logprob import fused_lm_head_logprob, fused_lm_head_ppo
from ..ops.ppo import PPOLossConfig, ppo_loss
from ..tpr.tree_plan_builder import SegmentObjectiveRef, TreeExecutionPlan


def batch_meta(batch: Any, key: str, default=None):
    """Non-tensor metadata from a dict, a TensorDict (non_tensor data) or an attribute."""
    getter = getattr(batch, "get_non_tensor", None)
    if callable(getter):
        try:
            return getter(key, default)
        except Exception:
            pass
    if isinstance(batch, dict):
        return batch.get(key, default)
    try:
        value = batch[key]
    except Exception:
        return getattr(batch, key, default)
    data = getattr(value, "data", None)
    return value if data is None or isinstance(value, Tensor) else data


def _rows(batch: Any, key: str) -> list[Tensor]:
    try:
        value = batch[key]
    except (KeyError, TypeError) as exc:
        raise ValueError(f"missing PPO field {key!r}") from exc
    rows = list(value) if isinstance(value, (list, tuple)) else list(value.unbind())
    if not all(isinstance(r, Tensor) and r.ndim == 1 for r in rows):
        raise ValueError(f"PPO field {key!r} must have 1-D rows")
    return rows


def _has(batch: Any, key: str) -> bool:
    try:
        return key in batch
    except TypeError:
        return False


@dataclass
class RefTable:
    """Flat per-ref arrays (host) of one tree, in ``objective_refs`` order."""

    segment_ids: Tensor
    query_offsets: Tensor
    targets: Tensor
    sample_rows: Tensor
    response_offsets: Tensor
    flat_index: Tensor      # index into the mini-batch flat PPO arrays


class SegmentPPOObjectiveAdapter:
    """Maps physical segment rows to logical PPO tokens and evaluates the PPO loss."""

    def __init__(self, batch: Any, loss_function: Callable | None = None, *, config: PPOLossConfig | None = None,
                 calculate_entropy: bool | None = None, dp_group: Any = None,
                 log_prob_chunk_size: int | None = None, device=None) -> None:
        cfg = getattr(loss_function, "keywords", {}).get("config") if loss_function is not None else None
        if cfg is not None:
            mode = cfg.policy_loss.get("loss_mode", "vanilla")
            if mode != "vanilla" or cfg.loss_agg_mode != "token-mean":
                raise NotImplementedError("segment-local PPO requires vanilla policy loss and token-mean aggregation, "
                                          f"got {mode!r} and {cfg.loss_agg_mode!r}")
        self.batch = batch
        self.loss_function = loss_function
        self.config = config or PPOLossConfig()
        self.calculate_entropy = bool(batch_meta(batch, "calculate_entropy", False)) if calculate_entropy is None \
            else bool(calculate_entropy)
        self.dp_group = dp_group
        if log_prob_chunk_size is not None and (not isinstance(log_prob_chunk_size, int)
                                                or isinstance(log_prob_chunk_size, bool) or log_prob_chunk_size <= 0):
            raise ValueError(f"log_prob_chunk_size must be a positive integer or None, got {log_prob_chunk_size!r}")
        self.log_prob_chunk_size = log_prob_chunk_size or 4096
        denom = batch_meta(batch, "batch_num_tokens", None)
        if denom is None:
            raise ValueError("PPO global batch_num_tokens is missing; compute it before TPR routing")
        self.dp_size = int(batch_meta(batch, "dp_size", 1) or 1)
        self.denominator = float(denom) / float(self.dp_size)
        self.capture_log_probs = bool(batch_meta(batch, "tpr_capture_log_probs", False))
        self.debug_new_log_probs: dict[tuple[int, int], float] = {}
        self._flat = self._flatten_ppo_inputs()
        self._device_flat: dict[str, Tensor] | None = None
        self.device = device

    # ------------------------------------------------------------------ host prep
    def _flatten_ppo_inputs(self):
        masks = _rows(self.batch, "response_mask")
        old = _rows(self.batch, "old_log_probs")
        adv = _rows(self.batch, "advantages")
        opt = {k: _rows(self.batch, k) for k in ("rollout_is_weights", "ref_log_prob") if _has(self.batch, k)}
        if len(old) != len(masks) or len(adv) != len(masks):
            raise ValueError("old_log_probs/advantages rows must match response_mask rows")
        offsets = [0]
        for m in masks:
            offsets.append(offsets[-1] + m.numel())
        flat = {
            "old_log_probs": torch.cat([r.detach().float().cpu() for r in old]),
            "advantages": torch.cat([r.detach().float().cpu() for r in adv]),
            "mask": torch.cat([m.detach().to(torch.bool).cpu() for m in masks]),
        }
        for k, rows in opt.items():
            flat[k] = torch.cat([r.detach().float().cpu() for r in rows])
        temp = batch_meta(self.batch, "temperature", 1.0)
        n = len(masks)
        if isinstance(temp, Tensor):
            t = temp.detach().float().cpu().flatten()
            t = t.expand(n).clone() if t.numel() == 1 else t
        elif isinstance(temp, (list, tuple)):
            t = torch.tensor([float(x) for x in temp])
        elif isinstance(temp, (int, float)):
            t = torch.full((n,), float(temp))
        else:
            raise TypeError(f"unsupported per-sample temperature type: {type(temp)!r}")
        if t.numel() != n or not bool(((t > 0) & torch.isfinite(t)).all()):
            raise ValueError("temperature must be finite and positive per row")
        self.row_offsets = offsets
        self._row_offsets_np = np.asarray(offsets, dtype=np.int64)
        self.row_temperature = t
        return flat

    def device_flat(self, device) -> dict[str, Tensor]:
        if self._device_flat is None:
            self._device_flat = {k: v.to(device, non_blocking=True) for k, v in self._flat.items()}
        return self._device_flat

    def ref_table(self, refs: Sequence[SegmentObjectiveRef]) -> RefTable:
        n = len(refs)
        cols = getattr(refs, "columns", None)
        if cols is not None:          # columnar refs: no per-ref Python objects
            cols = cols.T
        else:                         # one vectorised conversion (a per-element tensor write is a host op)
            cols = np.fromiter((x for r in refs for x in (r.segment_id, r.query_offset, r.target_token_id,
                                                          r.sample_row, r.response_offset)),
                               dtype=np.int64, count=5 * n).reshape(n, 5).T
        flat = self._row_offsets_np[cols[3]] + cols[4]
        a = torch.from_numpy(np.vstack([cols, flat[None]]))
        if n and not bool(self._flat["mask"][a[5]].all()):
            raise ValueError("objective ref points to a masked token")
        return RefTable(a[0], a[1], a[2], a[3], a[4], a[5])

    # ------------------------------------------------------------------ loss on selected rows
    def rows_loss(self, model, hidden: Tensor, local_rows: Tensor, table_targets: Tensor, sample_rows: Tensor,
                  flat_index: Tensor, *, host_keys: list[tuple] | None = None,
                  grad_scale: float | None = None) -> tuple[Tensor, dict]:
        """PPO loss of refs whose predicting query rows are ``hidden[local_rows]``.

        ``local_rows``, ``table_targets`` etc. are host tensors (one entry per ref).
        Dedupe on (row, target, temperature) happens here on the host.  With ``grad_scale`` (the
        factor the caller's backward applies to this loss) the CUDA path runs the LM-head backward
        inside the forward (:func:`~bridge_b200.ops.logprob.fused_lm_head_ppo`), so no logits are
        kept until backward.
        """
        dev = hidden.device
        temps = self.row_temperature[sample_rows]
        key = torch.stack([local_rows, table_targets, (temps * 1e6).round().long()], dim=1)
        uniq, inverse = torch.unique(key, dim=0, return_inverse=True)
        u_rows = uniq[:, 0]
        u_targets = uniq[:, 1]
        u_temps = torch.zeros(uniq.shape[0])
        u_temps[inverse] = temps
        pack = torch.stack([u_rows, u_targets]).to(dev, non_blocking=True)
        aux = torch.stack([inverse, flat_index]).to(dev, non_blocking=True)
        u_t = u_temps.to(dev, non_blocking=True)
        h = hidden.index_select(0, pack[0])
        flat = self.device_flat(dev)
        if grad_scale is not None and on_gpu(hidden):
            old = flat["old_log_probs"].index_select(0, aux[1])
            adv = flat["advantages"].index_select(0, aux[1])
            w = flat["rollout_is_weights"].index_select(0, aux[1]) if "rollout_is_weights" in flat else None
            c = self.config
            loss, stats, lp_u, ent_u = fused_lm_head_ppo(
                model.head_input(h), model.head_weight, pack[1], u_t, aux[0], old, adv, w, denom=self.denominator,
                clip_low=c.clip_ratio_low, clip_high=c.clip_ratio_high, clip_c=c.clip_ratio_c,
                vocab_start=model.vocab_start, tp_group=model.tp_group, with_entropy=self.calculate_entropy,
                chunk_rows=self.log_prob_chunk_size, grad_scale=grad_scale)
            metrics = {"n": int(local_rows.numel()), "stats": stats}
            if ent_u is not None:
                metrics["entropy_sum"] = ent_u.index_select(0, aux[0]).sum()
            if self.capture_log_probs:
                metrics["log_probs"] = lp_u.index_select(0, aux[0])
            return loss, metrics
        lp_u, ent_u = fused_lm_head_logprob(model.head_input(h), model.head_weight, pack[1], u_t,
                                            vocab_start=model.vocab_start, tp_group=model.tp_group,
                                            with_entropy=self.calculate_entropy,
                                            chunk_rows=self.log_prob_chunk_size)
        lp = lp_u.index_select(0, aux[0])
        old = flat["old_log_probs"].index_select(0, aux[1])
        adv = flat["advantages"].index_select(0, aux[1])
        w = flat["rollout_is_weights"].index_select(0, aux[1]) if "rollout_is_weights" in flat else None
        loss, stats = ppo_loss(lp, old, adv, denom=self.denominator, cfg=self.config, weights=w)
        metrics = {"n": int(local_rows.numel()), "stats": stats}
        if ent_u is not None:
            metrics["entropy_sum"] = ent_u.index_select(0, aux[0]).detach().sum()
        if self.capture_log_probs:
            metrics["log_probs"] = lp.detach()
        return loss, metrics

    # ------------------------------------------------------------------ per-segment API
    def bind_tree(self, tree_plan: TreeExecutionPlan, *, shard_for_segment=None, model=None):
        """Return ``(segment_loss_fn, per_segment_ref_counts)`` for one tree."""
        if not isinstance(tree_plan, TreeExecutionPlan):
            raise TypeError("tree_plan must be a TreeExecutionPlan")
        by_seg: dict[int, list[SegmentObjectiveRef]] = {s: [] for s in tree_plan.segment_plan.segments}
        for ref in tree_plan.objective_refs:
            by_seg[ref.segment_id].append(ref)
        if not tree_plan.objective_refs:
            raise ValueError("tree has no supervised logical response tokens")
        if shard_for_segment is not None:
            for sid, refs in by_seg.items():
                shard = shard_for_segment(tree_plan.segment_plan.get(sid))
                by_seg[sid] = [r for r in refs if shard.owns(r.query_offset)]
        counts = {sid: len(r) for sid, r in by_seg.items()}

        def segment_loss_fn(segment, outputs):
            shard = None if shard_for_segment is None else shard_for_segment(segment)
            return self.compute_loss(segment, outputs, by_seg[segment.segment_id], shard=shard, model=model)

        return segment_loss_fn, counts

    def compute_loss(self, segment, outputs, refs: Sequence[SegmentObjectiveRef], *, shard=None, model=None):
        """``outputs`` is the segment's final hidden states ``[local_len, hidden]`` (or an object with ``.hidden``)."""
        refs = tuple(refs)
        if not refs:
            raise ValueError("no objective refs: use a zero-gradient relay path for this segment")
        hidden = getattr(outputs, "hidden", outputs)
        model = getattr(outputs, "model", model)
        if model is None:
            raise ValueError("compute_loss needs the model (LM head) to project the selected rows")
        want = segment.length if shard is None else shard.local_length
        if hidden.ndim != 2 or hidden.shape[0] != want:
            raise ValueError(f"expected hidden states [{want}, hidden], got {tuple(hidden.shape)}")
        rows = []
        for r in refs:
            if r.segment_id != segment.segment_id:
                raise ValueError("objective ref belongs to another segment")
            if not 0 <= r.query_offset < segment.length:
                raise ValueError("objective ref query_offset is outside segment")
            off = r.query_offset if shard is None else shard.global_to_local(r.query_offset)
            if off is None:
                raise ValueError("PPO ref is not owned by this CP rank")
            rows.append(off)
        tab = self.ref_table(refs)
        loss, metrics = self.rows_loss(model, hidden, torch.tensor(rows, dtype=torch.long), tab.targets,
                                       tab.sample_rows, tab.flat_index)
        if self.capture_log_probs and "log_probs" in metrics:
            for r, v in zip(refs, metrics["log_probs"].float().cpu().tolist()):
                k = (r.sample_row, r.response_offset)
                if k in self.debug_new_log_probs:
                    raise ValueError(f"duplicate new_log_prob probe for logical token {k}")
                self.debug_new_log_probs[k] = v
        return loss, metrics
