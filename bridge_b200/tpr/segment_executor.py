"""Per-segment Push / Pop / VisitLeaf execution with relayed prefix gradients.

* **Push(s)** -- graph-free forward of ``s`` over its ancestors' KV; keeps the
  compact new K/V (and GDN final states) on the stack for descendants.
* **Pop(s)** -- recompute ``s`` with grad over fresh ancestor *anchors*, then one
  backward from ``[loss(s), new K/V of s, GDN final states of s]`` with the
  relayed ``[1, dK/dV, dState]`` accumulated by its children; the anchors'
  gradients are then added to the ancestors' accumulators.
* **VisitLeaf(s)** -- a leaf's adjacent Push/Pop fused: one forward, one backward.

Every CP rank runs the same autograd graph even with no owned loss term
(a connected zero loss), so ring/all-gather collectives never diverge.

This executor keeps the reference's one-segment-per-forward semantics (and is
the CP path).  :mod:`bridge_b200.tpr.forest_executor` is the batched engine
used by the training entry points on one GPU / per DP rank.

Parity: verl/models/mcore/tpr/segment_executor.py:85-877.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn.functional as F
from torch import Tensor, nn
from torch.utils.checkpoint import checkpoint

from .activation_offload import validate_activation_offload, with_activation_offload
from .context import KVPair, TPRAttentionContext, use_tpr_attention_context
from .kv_stack import KVStack
from .prefix_state import GDNLayerState, GDNPrefixAnchors, GDNPrefixState
from .rope import sharded_position_ids
from .segment_plan import SegmentId, SegmentLossTerm, SegmentPlan, SegmentSpec
from .shard import PrefixShard, SequenceShard


@dataclass(frozen=True, slots=True)
class SegmentForwardResult:
    segment_id: SegmentId
    prefix_length: int
    suffix_length: int
    layer_count: int


@dataclass(frozen=True, slots=True)
class SegmentBackwardResult:
    segment_id: SegmentId
    loss_sum: Tensor
    normalized_loss: Tensor
    loss_term_count: int
    relayed_layer_count: int


@dataclass(frozen=True, slots=True)
class LeafVisitResult:
    forward: SegmentForwardResult
    backward: SegmentBackwardResult


@dataclass(frozen=True, slots=True)
class SegmentOutputs:
    """What a segment forward hands to an external objective: final hidden rows + the model."""

    hidden: Tensor
    model: nn.Module


def model_device(model: nn.Module) -> torch.device:
    try:
        return next(model.parameters()).device
    except StopIteration as exc:
        raise ValueError("model must contain at least one parameter") from exc


class SegmentExecutor:
    """Graph-free Push and gradient-carrying Pop for one :class:`SegmentPlan`."""

    def __init__(self, model: nn.Module, plan: SegmentPlan, *, expected_layer_numbers=None,
                 kv_stack: KVStack | None = None, loss_scale_func: Callable[[Tensor], Tensor] | None = None,
                 loss_chunk_size: int | None = None, cp_group: Any = None, cp_backend: Any = None,
                 segment_loss_fn: Callable | None = None, segment_loss_term_counts: Mapping[int, int] | None = None,
                 activation_offload: Any = None) -> None:
        if not isinstance(model, nn.Module):
            raise TypeError(f"model must be torch.nn.Module, got {type(model).__name__}")
        if not isinstance(plan, SegmentPlan):
            raise TypeError(f"plan must be SegmentPlan, got {type(plan).__name__}")
        if expected_layer_numbers is None:
            expected_layer_numbers = getattr(model, "attention_layer_numbers", None)
            if expected_layer_numbers is None:
                raise ValueError("cannot infer TPR layer numbers; pass expected_layer_numbers explicitly")
        layers = tuple(expected_layer_numbers)
        if any(not isinstance(x, int) or isinstance(x, bool) or x <= 0 for x in layers):
            raise ValueError(f"expected_layer_numbers must contain positive integers, got {layers}")
        if len(set(layers)) != len(layers):
            raise ValueError(f"expected_layer_numbers contains duplicates: {layers}")
        if plan.topology_only != (segment_loss_fn is not None):
            raise ValueError("topology_only SegmentPlan requires segment_loss_fn; CE SegmentPlan must use the CE path")
        counts = dict(segment_loss_term_counts or {})
        if segment_loss_fn is not None:
            if not callable(segment_loss_fn):
                raise TypeError("segment_loss_fn must be callable")
            if not counts:
                raise ValueError("segment_loss_term_counts is required for external objectives")
            if any(s not in plan.segments or c < 0 for s, c in counts.items()):
                raise ValueError("invalid external segment objective counts")
        elif counts:
            raise ValueError("segment_loss_term_counts is only valid with segment_loss_fn")
        if loss_chunk_size is not None and (not isinstance(loss_chunk_size, int) or isinstance(loss_chunk_size, bool)
                                            or loss_chunk_size <= 0):
            raise ValueError(f"loss_chunk_size must be a positive integer or None, got {loss_chunk_size!r}")
        self.model = model
        self.plan = plan
        self.expected_layer_numbers = tuple(sorted(layers))
        self.kv_stack = KVStack() if kv_stack is None else kv_stack
        self.loss_scale_func = loss_scale_func
        self.loss_chunk_size = loss_chunk_size
        self.segment_loss_fn = segment_loss_fn
        self.segment_loss_term_counts = counts
        self.segment_loss_metrics: list[tuple[SegmentId, dict]] = []
        self.cp_group = cp_group
        self.gdn_layer_numbers = tuple(sorted(getattr(model, "gdn_layer_numbers", ()) or ()))
        if set(self.gdn_layer_numbers) & set(self.expected_layer_numbers):
            raise ValueError("expected_layer_numbers describes attention layers only, not GDN layers")
        self.gdn_states: dict[SegmentId, GDNPrefixState] = {}
        if cp_group is None:
            if cp_backend is not None and not isinstance(cp_backend, str):
                raise ValueError("cp_backend requires a cp_group")
            self.cp_size, self.cp_rank, self.cp_backend = 1, 0, None
        else:
            from ..parallel.backend import resolve_tpr_cp_backend
            from ..parallel.execution_context import resolve_cp_group

            self.cp_size, self.cp_rank = resolve_cp_group(cp_group)
            if self.cp_size <= 1:
                raise ValueError(f"cp_group must contain more than one rank, got {self.cp_size}")
            self.cp_backend = resolve_tpr_cp_backend(cp_backend, cp_group=cp_group, parallel_size=self.cp_size,
                                                     parallel_rank=self.cp_rank)
            if self.gdn_layer_numbers and self.cp_backend.backend_name != "ring":
                raise NotImplementedError("hybrid GDN TPR under CP requires the ring backend")
            for seg in plan.segments.values():
                try:
                    self.cp_backend.validate_segment_length(seg.length)
                except ValueError as exc:
                    raise ValueError(f"segment {seg.segment_id} {exc}") from exc
        self.activation_offload = activation_offload
        validate_activation_offload(model, self.cp_size, self.cp_backend, activation_offload)
        self._failed = False

    # ------------------------------------------------------------------ properties
    @property
    def failed(self) -> bool:
        return self._failed

    @property
    def cp_enabled(self) -> bool:
        return self.cp_group is not None

    def _healthy(self) -> None:
        if self._failed:
            raise RuntimeError("SegmentExecutor is failed and cannot continue")

    # ------------------------------------------------------------------ events
    def push(self, segment_id: SegmentId) -> SegmentForwardResult:
        """Graph-free forward; saves compact KV / GDN states. No loss is computed."""
        self._healthy()
        try:
            seg = self.plan.get(segment_id)
            past = {} if self.cp_enabled else self.kv_stack.build_past_key_values()
            ctx, hidden = self._forward(seg, past_key_values=past, no_grad=True)
            del hidden
            self._assert_layers(ctx)
            kv = {layer: (k.detach().clone(memory_format=torch.contiguous_format),
                          v.detach().clone(memory_format=torch.contiguous_format))
                  for layer, (k, v) in ctx.new_key_values.items()}
            if self.gdn_layer_numbers:
                self.gdn_states[segment_id] = GDNPrefixState.save(segment_id, seg.length, ctx.new_gdn_states)
            n_layers = len(kv) + len(ctx.new_gdn_states)
            del ctx
            self.kv_stack.push(seg, kv, shard=self._shard(seg))
            return SegmentForwardResult(segment_id, seg.prefix_length, seg.length, n_layers)
        except Exception:
            self._failed = True
            raise

    @with_activation_offload
    def pop(self, segment_id: SegmentId) -> SegmentBackwardResult:
        """Recompute with grad and back-propagate owned loss + relayed KV/GDN gradients."""
        self._healthy()
        try:
            top = self.kv_stack.top()
            if top.segment.segment_id != segment_id:
                raise RuntimeError(f"cannot pop segment {segment_id}: stack top is {top.segment.segment_id}")
            relayed = dict(top.kv.consume_gradients())
            if relayed and tuple(relayed) != self.expected_layer_numbers:
                raise RuntimeError(f"segment {segment_id} relayed KV gradient layers must be "
                                   f"{self.expected_layer_numbers}, got {tuple(relayed)}")
            entry = self.kv_stack.pop(segment_id)
            seg = entry.segment
            gdn = self.gdn_states.pop(segment_id) if self.gdn_layer_numbers else None
            relayed_gdn = {} if gdn is None else dict(gdn.consume_gradients())
            entry.kv.release()  # the recompute below regenerates this segment's KV with a graph
            anchors, past = self._ancestor_anchors()
            gdn_parent, gdn_anchors = self._gdn_parent_anchors()
            ctx, hidden = self._forward(seg, past_key_values=past, no_grad=False,
                                        sharded_anchors=anchors if self.cp_enabled else None,
                                        initial_gdn_states={} if gdn_anchors is None else gdn_anchors.layer_states)
            self._assert_layers(ctx)
            loss_sum, normalized = self._compute_loss(seg, hidden)
            owned = self._owned_count(seg)
            roots: list[Tensor] = []
            grads: list[Tensor | None] = []
            if owned or self.cp_enabled:
                roots.append(self._backward_loss(normalized, hidden, owned > 0))
                grads.append(None)
            for layer in self.expected_layer_numbers:
                if layer in relayed:
                    k, v = ctx.new_key_values[layer]
                    roots += [k, v]
                    grads += list(relayed[layer])
            for layer, g in relayed_gdn.items():
                st = ctx.new_gdn_states[layer]
                roots += [st.conv_state, st.recurrent_state]
                grads += [g.conv_state, g.recurrent_state]
            if roots:
                torch.autograd.backward(roots, grad_tensors=grads)
                self._accumulate_anchor_grads(anchors)
                if gdn_anchors is not None:
                    gdn_parent.accumulate_anchor_gradients(gdn_anchors)
            if gdn is not None:
                gdn.release()
            return SegmentBackwardResult(segment_id, loss_sum.detach(), normalized.detach(), owned,
                                         len(relayed) + len(relayed_gdn))
        except Exception:
            self._failed = True
            raise

    @with_activation_offload
    def visit_leaf(self, segment_id: SegmentId) -> LeafVisitResult:
        """One forward + one backward of a leaf; nothing is pushed."""
        self._healthy()
        try:
            seg = self.plan.get(segment_id)
            if self.plan.child_ids(segment_id):
                raise ValueError(f"segment {segment_id} is not a leaf")
            parent = self.kv_stack.top().segment.segment_id if len(self.kv_stack) else None
            if seg.parent_id != parent:
                raise RuntimeError(f"cannot visit leaf {segment_id}: expected parent on stack {seg.parent_id}, "
                                   f"got {parent}")
            if seg.prefix_length != self.kv_stack.prefix_length:
                raise RuntimeError(f"cannot visit leaf {segment_id}: stack prefix length is "
                                   f"{self.kv_stack.prefix_length}, got {seg.prefix_length}")
            anchors, past = self._ancestor_anchors()
            gdn_parent, gdn_anchors = self._gdn_parent_anchors()
            ctx, hidden = self._forward(seg, past_key_values=past, no_grad=False,
                                        sharded_anchors=anchors if self.cp_enabled else None,
                                        initial_gdn_states={} if gdn_anchors is None else gdn_anchors.layer_states,
                                        capture_gdn_final_state=False)
            self._assert_layers(ctx, gdn=False)
            loss_sum, normalized = self._compute_loss(seg, hidden)
            owned = self._owned_count(seg)
            torch.autograd.backward(self._backward_loss(normalized, hidden, owned > 0))
            self._accumulate_anchor_grads(anchors)
            if gdn_anchors is not None:
                gdn_parent.accumulate_anchor_gradients(gdn_anchors)
            fwd = SegmentForwardResult(segment_id, seg.prefix_length, seg.length,
                                       len(ctx.new_key_values) + len(self.gdn_layer_numbers))
            return LeafVisitResult(fwd, SegmentBackwardResult(segment_id, loss_sum.detach(), normalized.detach(),
                                                              owned, 0))
        except Exception:
            self._failed = True
            raise

    # ------------------------------------------------------------------ internals
    def _shard(self, seg: SegmentSpec) -> SequenceShard:
        if not self.cp_enabled:
            return PrefixShard.full(seg.length)
        return self.cp_backend.make_sequence_shard(seg.length)

    def _ancestor_anchors(self):
        if self.cp_enabled:
            from ..parallel.execution_context import build_sharded_past_anchors

            return build_sharded_past_anchors(self.kv_stack), {}
        anchors = self.kv_stack.build_past_anchors()
        return anchors, anchors.key_values

    def _accumulate_anchor_grads(self, anchors) -> None:
        if self.cp_enabled:
            from ..parallel.execution_context import accumulate_sharded_past_anchor_gradients

            accumulate_sharded_past_anchor_gradients(self.kv_stack, anchors)
        elif anchors.key_values:
            self.kv_stack.accumulate_anchor_gradients(anchors)

    def _gdn_parent_anchors(self) -> tuple[GDNPrefixState | None, GDNPrefixAnchors | None]:
        if not self.gdn_layer_numbers or not len(self.kv_stack):
            return None, None
        parent = self.gdn_states[self.kv_stack.top().segment.segment_id]
        return parent, parent.make_anchors()

    def _forward(self, seg: SegmentSpec, *, past_key_values, no_grad: bool, sharded_anchors=None,
                 initial_gdn_states=None, capture_gdn_final_state: bool = True):
        dev = model_device(self.model)
        shard = self._shard(seg)
        ids = shard.select(seg.token_ids).to(dev, non_blocking=True)
        pos = sharded_position_ids(seg.position_start, shard).to(dev, non_blocking=True)
        backend = None
        if self.cp_enabled:
            backend = self.cp_backend.make_attention_backend(self.kv_stack,
                                                             expected_layer_numbers=self.expected_layer_numbers,
                                                             current_shard=shard, past_anchors=sharded_anchors)
        if initial_gdn_states is None and self.gdn_layer_numbers and len(self.kv_stack):
            initial_gdn_states = self.gdn_states[self.kv_stack.top().segment.segment_id].layer_states
        ctx = TPRAttentionContext(prefix_length=seg.prefix_length, suffix_length=seg.length,
                                  past_key_values=past_key_values, position_ids=pos, attention_backend=backend,
                                  initial_gdn_states=initial_gdn_states or {},
                                  capture_gdn_final_state=capture_gdn_final_state)
        with (torch.no_grad() if no_grad else torch.enable_grad()), use_tpr_attention_context(ctx):
            hidden = self.model(ids, pos, seg.position_end)
        if hidden.ndim != 2 or hidden.shape[0] != shard.local_length:
            raise ValueError(f"model must return hidden [local_length={shard.local_length}, hidden], "
                             f"got {tuple(hidden.shape)}")
        return ctx, hidden

    def _owned_terms(self, seg: SegmentSpec) -> tuple[SegmentLossTerm, ...]:
        if not self.cp_enabled:
            return seg.loss_terms
        shard = self._shard(seg)
        return tuple(t for t in seg.loss_terms if shard.owns(t.query_offset))

    def _owned_count(self, seg: SegmentSpec) -> int:
        if self.segment_loss_fn is not None:
            return self.segment_loss_term_counts.get(seg.segment_id, 0)
        return len(self._owned_terms(seg))

    def _compute_loss(self, seg: SegmentSpec, hidden: Tensor) -> tuple[Tensor, Tensor]:
        if self.segment_loss_fn is not None:
            if not self._owned_count(seg):
                z = hidden.float().sum() * 0.0
                return z, z
            loss, metrics = self.segment_loss_fn(seg, SegmentOutputs(hidden, self.model))
            if not isinstance(loss, Tensor) or loss.numel() != 1 or not loss.requires_grad:
                raise TypeError("external segment objective must return a differentiable scalar Tensor")
            self.segment_loss_metrics.append((seg.segment_id, metrics))
            return loss, loss
        terms = self._owned_terms(seg)
        if not terms:
            z = hidden.new_zeros((), dtype=torch.float32)
            return z, z
        shard = self._shard(seg)
        offs = [shard.global_to_local(t.query_offset) for t in terms]
        if any(o is None for o in offs):
            raise RuntimeError(f"segment {seg.segment_id} has a loss term outside its local shard")
        vocab = getattr(self.model, "vocab_size", None)
        top = max(t.target_token_id for t in terms)
        if vocab is not None and top >= vocab:
            raise ValueError(f"segment {seg.segment_id} target token {top} is outside vocabulary size {vocab}")
        dev = hidden.device
        rows = torch.tensor(offs, dtype=torch.long, device=dev)
        targets = torch.tensor([t.target_token_id for t in terms], dtype=torch.long, device=dev)
        weights = torch.tensor([t.weight for t in terms], dtype=torch.float32, device=dev)
        chunk = self.loss_chunk_size or len(terms)
        parts = []
        for s in range(0, len(terms), chunk):
            e = min(len(terms), s + chunk)
            if self.loss_chunk_size is not None and len(terms) > chunk:
                parts.append(checkpoint(self._ce_rows, hidden, rows[s:e], targets[s:e], use_reentrant=False,
                                        preserve_rng_state=False))
            else:
                parts.append(self._ce_rows(hidden, rows[s:e], targets[s:e]))
        per_term = torch.cat(parts)
        loss_sum = (per_term.float() * weights).sum()
        return loss_sum, loss_sum / self.plan.total_loss_weight

    def _ce_rows(self, hidden: Tensor, rows: Tensor, targets: Tensor) -> Tensor:
        from ..ops.logprob import fused_lm_head_logprob

        h = hidden.index_select(0, rows)
        ones = torch.ones(rows.shape[0], device=h.device)
        lp, _ = fused_lm_head_logprob(self.model.head_input(h), self.model.head_weight, targets, ones,
                                      vocab_start=self.model.vocab_start, tp_group=self.model.tp_group)
        return -lp

    def _backward_loss(self, normalized: Tensor, hidden: Tensor, has_owned: bool) -> Tensor:
        loss = normalized * self.cp_size if has_owned else hidden.float().sum() * 0.0
        return loss if self.loss_scale_func is None else self.loss_scale_func(loss)

    def _assert_layers(self, ctx: TPRAttentionContext, *, gdn: bool = True) -> None:
        ctx.assert_new_kv_layers(self.expected_layer_numbers)
        ctx.assert_new_gdn_layers(self.gdn_layer_numbers if gdn else ())
