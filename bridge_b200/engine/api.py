"""Public TPR entry points: module-spec install, CE request entry, PPO mini-batch entry.

* :func:`run_tpr_forward_backward_batch` -- PPO mini-batch -> token-trie forest
  -> batched level execution (under CP: segment-granular placement over the CP
  group, or per-tree Push/Pop with the named CP backend when a segment is longer
  than one rank's token budget) -> one gradient finalisation; returns
  ``{"model_output", "loss", "metrics"}`` like verl.
* :func:`run_tpr_forward_backward` -- CE request (a :class:`SegmentPlan` with
  loss terms, optional fixed event order) through one SegmentExecutor.

Parity: verl/models/mcore/tpr/megatron_adapter.py:37-529 and
verl/models/mcore/tpr/engine_adapter.py:24-39 (TPR_REQUEST_KEY,
TPRForwardBackwardRequest), verl/models/mcore/tpr/module_spec.py:34-131.
"""

from __future__ import annotations

import os
import time
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any

import torch
from torch import Tensor, nn

from ..models.layers import TPRGatedDeltaNet, TPRSelfAttention
from ..rl.objective import SegmentPPOObjectiveAdapter, batch_meta
from ..tpr.forest_executor import ForestExecutor
from ..tpr.scheduler import FixedTopologyScheduler, TPRBatchRunner
from ..tpr.segment_executor import SegmentExecutor
from ..tpr.segment_plan import SegmentEvent, SegmentPlan
from ..tpr.tree_plan_builder import build_tree_execution_plans

TPR_REQUEST_KEY = "tpr_forward_backward_request"


@dataclass(frozen=True, slots=True)
class TPRForwardBackwardRequest:
    plan: SegmentPlan
    events: tuple[SegmentEvent, ...] | None = None

    def __post_init__(self) -> None:
        if not isinstance(self.plan, SegmentPlan):
            raise TypeError("plan must be a SegmentPlan")
        if self.plan.topology_only:
            raise ValueError("a CE request needs a plan with loss terms (not topology_only)")
        if self.events is not None:
            object.__setattr__(self, "events", self.plan.validate_events(self.events))


# --------------------------------------------------------------------------- module spec
def replace_self_attention_with_tpr(model: nn.Module) -> nn.Module:
    """Validate that every token-mixing layer is TPR-capable (this framework builds them natively).

    A foreign attention module (anything that is neither ``TPRSelfAttention``
    nor ``TPRGatedDeltaNet``) cannot take external prefix state and is rejected.
    """
    layers = getattr(model, "layers", None)
    if layers is None:
        raise TypeError("model has no decoder layers")
    for layer in layers:
        mixer = getattr(layer, "self_attention", None)
        if not isinstance(mixer, (TPRSelfAttention, TPRGatedDeltaNet)):
            raise TypeError(f"layer {getattr(layer, 'layer_number', '?')} uses {type(mixer).__name__}, "
                            "which cannot consume TPR prefix state")
    return model


def make_tpr_module_spec_provider(provider: Callable[[], nn.Module]) -> Callable[[], nn.Module]:
    def build() -> nn.Module:
        return replace_self_attention_with_tpr(provider())

    build.tpr_installed = True  # type: ignore[attr-defined]
    return build


def install_tpr_module_spec(provider: Callable[[], nn.Module]) -> Callable[[], nn.Module]:
    if getattr(provider, "tpr_installed", False):
        return provider
    return make_tpr_module_spec_provider(provider)


# --------------------------------------------------------------------------- helpers
def validate_tpr_parallel_sizes(sizes: dict[str, int], *, ppo: bool) -> int:
    if sizes.get("PP", 1) != 1:
        raise NotImplementedError("TPR does not support pipeline parallelism")
    for k, v in sizes.items():
        if not isinstance(v, int) or v < 1:
            raise ValueError(f"{k} size must be a positive integer, got {v!r}")
    return sizes.get("TP", 1)


def trajectory_keys_from_minibatch(data: Any) -> tuple[str, ...]:
    keys = batch_meta(data, "tpr_trajectory_keys", None)
    if keys is not None:
        keys = tuple(str(k) for k in keys)
        if len(set(keys)) != len(keys):
            raise ValueError("tpr_trajectory_keys must be unique")
        return keys
    uids = batch_meta(data, "uid", None)
    if uids is None:
        raise ValueError("TPR PPO needs tpr_trajectory_keys or uid to group trajectories")
    out = []
    for row, u in enumerate(uids):
        if hasattr(u, "item"):
            u = u.item()
        if isinstance(u, bytes):
            u = u.decode("utf-8")
        if not isinstance(u, (str, int)) or not str(u):
            raise ValueError(f"uid row {row} must be a nonempty string or integer")
        out.append(f"{u}_tpr_{row}")
    return tuple(out)


def _rows(data, key):
    v = data[key]
    return list(v) if isinstance(v, (list, tuple)) else list(v.unbind())


# --------------------------------------------------------------------------- CE entry
def run_tpr_forward_backward(engine, request: TPRForwardBackwardRequest) -> dict:
    if not isinstance(request, TPRForwardBackwardRequest):
        raise TypeError("request must be a TPRForwardBackwardRequest")
    from ..parallel.engine_runtime import aggregate_cp_loss, resolve_engine_cp_runtime

    model = engine.model
    rt = resolve_engine_cp_runtime(engine)
    ex = SegmentExecutor(model, request.plan, cp_group=rt.group, cp_backend=rt.backend,
                         loss_chunk_size=engine.engine_config.log_prob_chunk_tokens or None)
    sched = FixedTopologyScheduler(request.plan, ex, events=request.events)
    result = sched.run()
    engine.finalize_model_grads()
    loss_sum, loss = aggregate_cp_loss(result.loss_sum, result.normalized_loss, rt)
    return {
        "tpr_loss": float(loss.item()),
        "tpr_loss_sum": float(loss_sum.item()),
        "tpr_cp_size": rt.size,
        "tpr_cp_backend": None if rt.backend is None else rt.backend.backend_name,
        "tpr_peak_path_tokens": result.peak_path_tokens,
        "tpr_segment_count": result.executed_segment_count,
        "tpr_direct_leaf_count": result.direct_leaf_count,
    }


# --------------------------------------------------------------------------- PPO entry
@dataclass
class PreparedTPRBatch:
    """Host-side product of planning one PPO mini-batch (reusable across identical steps)."""

    data: Any
    forest: Any
    objective: SegmentPPOObjectiveAdapter
    logical_input_tokens: int
    stage_ms: dict
    nodes: Any = None


def prepare_tpr_batch(engine, data: Any, loss_function: Any = None) -> PreparedTPRBatch:
    """Validate the mini-batch, build the token-trie forest and the PPO ref tables (host work)."""
    ec = engine.engine_config
    if not ec.tpr_enabled:
        raise RuntimeError("TPR PPO requires engine_config.tpr_enabled=True at model creation")
    ps = engine.parallel
    validate_tpr_parallel_sizes({"TP": ps.tp, "CP": ps.cp, "DP": ps.dp, "EP": ps.ep, "PP": 1}, ppo=True)
    token_count = batch_meta(data, "batch_num_tokens", None)
    dp_size = batch_meta(data, "dp_size", None)
    if token_count is None or int(token_count) <= 0 or int(dp_size or 0) != ps.dp:
        raise ValueError(f"engine must attach positive GLOBAL batch_num_tokens and the actual dp_size={ps.dp}")
    t0 = time.perf_counter()
    keys = trajectory_keys_from_minibatch(data)
    forest = build_tree_execution_plans(keys, data, tree_policy=ec.tree_policy,
                                        turn_min_segment_tokens=ec.turn_min_segment_tokens)
    if not forest.trees or not forest.logical_loss_tokens:
        raise ValueError("TPR PPO mini-batch has no supervised response tokens")
    stage = {"tree_build_cpu_ms": (time.perf_counter() - t0) * 1e3}
    if ps.tp > 1:
        from ..tpr.tp_validation import assert_tp_plan_agreement, digest_forest_plan

        assert_tp_plan_agreement(digest_forest_plan(forest), tp_size=ps.tp, group=ps.tp_group)
    objective = SegmentPPOObjectiveAdapter(data, loss_function, dp_group=ps.dp_group,
                                           log_prob_chunk_size=ec.log_prob_chunk_tokens or None)
    logical_inputs = sum(int(r.numel()) for r in _rows(data, "input_ids"))
    return PreparedTPRBatch(data, forest, objective, logical_inputs, stage)


def offload_config(ec):
    """``EngineConfig.activation_offload`` as the executors' offload config (None when off)."""
    if not ec.activation_offload:
        return None
    from ..tpr.activation_offload import OffloadConfig

    return OffloadConfig(enabled=True)


def max_segment_tokens(forest) -> int:
    return max((s.length for t in forest.trees for s in t.segment_plan.segments.values()), default=0)


def forest_fits(engine, forest, rt) -> bool:
    """Whether the batched forest executor runs this forest (``executor="forest"``, the default).  It
    runs any forest, on one rank or under CP: a segment longer than one rank's token budget becomes a
    chain of budget-sized pieces (each the prefix of the next).  ``executor="segment"`` selects the
    per-tree executor, which splits every segment over the CP group with the configured backend."""
    return engine.engine_config.executor == "forest"


def execute_prepared_tpr_batch(engine, prepared: PreparedTPRBatch, *, sync_loss: bool = True) -> dict:
    """Run the forest schedule of a prepared mini-batch and finalise gradients once."""
    from ..parallel.engine_runtime import aggregate_cp_loss, resolve_engine_cp_runtime

    ec = engine.engine_config
    model = engine.model
    if not model.training:
        raise RuntimeError("TPR PPO requires model.train()")
    forest, objective = prepared.forest, prepared.objective
    objective._device_flat = None  # re-stage the per-ref PPO inputs (one H2D copy per step)
    rt = resolve_engine_cp_runtime(engine)
    t_run = time.perf_counter()
    metrics: dict[str, Any] = {}
    profiler = None
    if ec.exec_profile:
        from ..utils.profiler import SegmentEventProfiler

        profiler = SegmentEventProfiler()
        engine._tpr_segment_event_profiler = profiler
    if forest_fits(engine, forest, rt):
        cp = None
        if rt.group is not None:
            cp = getattr(engine, "_tpr_forest_cp", None)
            if cp is None or cp.group is not rt.group:
                from ..parallel.forest_cp import ForestCP

                cp = engine._tpr_forest_cp = ForestCP(rt.group, comm=ec.cp_comm)
        fx = ForestExecutor(model, objective, mode=ec.forest_mode, token_budget=ec.token_budget,
                            loss_scale=float(rt.size), cp=cp, offload=offload_config(ec))
        # the data-parallel reduction of each layer's gradients starts as soon as the step's last
        # backward has finished that layer (sharded NVLink optimizer)
        fx.before_final_backward = getattr(engine.optimizer, "arm_overlap", None)
        fx.profiler = profiler
        if prepared.nodes is None:
            prepared.nodes = fx.plan(forest)
        res = fx.run(forest, prepared.nodes)
        if sync_loss and not bool(torch.isfinite(res.normalized_loss).item()):
            raise FloatingPointError("non-finite TPR PPO loss; gradients will not be finalized")
        engine.finalize_model_grads()
        total_loss, stats = res.normalized_loss, res.stats
        metrics["tpr/forward_tokens"] = [res.forward_tokens]
        metrics["tpr/backward_tokens"] = [res.backward_tokens]
        metrics["tpr/chunks"] = [res.chunks]
        if fx.offload is not None:
            metrics["tpr/offloaded_bytes"] = [fx.offloaded_bytes]
        if objective.calculate_entropy and "entropy_sum" in res.metrics:
            metrics["actor/entropy"] = [res.metrics["entropy_sum"] / forest.logical_loss_tokens]
    else:
        shard_for = None if rt.backend is None else (lambda seg: rt.backend.make_sequence_shard(seg.length))
        seg_stats = []

        def run_tree(tree_plan):
            fn, counts = objective.bind_tree(tree_plan, shard_for_segment=shard_for, model=model)
            ex = SegmentExecutor(model, tree_plan.segment_plan, segment_loss_fn=fn, segment_loss_term_counts=counts,
                                 cp_group=rt.group, cp_backend=rt.backend, activation_offload=offload_config(ec))
            out = FixedTopologyScheduler(tree_plan.segment_plan, ex, event_profiler=profiler,
                                         tree_index=len(seg_stats)).run()
            if sync_loss and not bool(torch.isfinite(out.normalized_loss).item()):
                raise FloatingPointError("non-finite TPR PPO tree loss; gradients will not be finalized")
            seg_stats.extend(m for _, m in ex.segment_loss_metrics)
            return out

        res = TPRBatchRunner(run_tree=run_tree, finalize_gradients=engine.finalize_model_grads).run(forest)
        total_loss = res.normalized_loss
        rows = [m["stats"] * m["n"] for m in seg_stats]
        stats = torch.stack(rows).sum(0) / max(sum(m["n"] for m in seg_stats), 1) if rows else None
    stage = dict(prepared.stage_ms)
    stage["tree_run_and_finalize_host_ms"] = (time.perf_counter() - t_run) * 1e3
    _, global_loss = aggregate_cp_loss(total_loss, total_loss, rt)
    unique = forest.unique_tokens
    metrics.update({
        "tpr/forest_trees": [len(forest.trees)],
        "tpr/physical_segments": [forest.segment_count],
        "tpr/logical_loss_tokens": [forest.logical_loss_tokens],
        "tpr/logical_input_tokens": [prepared.logical_input_tokens],
        "tpr/unique_tree_tokens": [unique],
        "tpr/topology_token_reuse_ratio": [prepared.logical_input_tokens / unique],
    })
    if stats is not None:
        names = ("actor/pg_clipfrac", "actor/pg_clipfrac_lower", "actor/ppo_kl", "actor/ratio_mean")
        metrics.update({n: [stats[i]] for i, n in enumerate(names)})
    if sync_loss:
        loss_val: Any = float(global_loss.item())
        if loss_val != loss_val or loss_val in (float("inf"), float("-inf")):
            raise FloatingPointError("non-finite TPR PPO mini-batch loss")
        for k, v in metrics.items():
            metrics[k] = [float(x.item()) if isinstance(x, Tensor) else float(x) for x in v]
    else:
        loss_val = global_loss
    if ec.exec_profile:
        engine._tpr_stage_profile = stage
    return {"model_output": {}, "loss": [loss_val], "metrics": metrics}


def run_tpr_forward_backward_batch(engine, data: Any, loss_function: Any = None, *, forward_only: bool = False,
                                   sync_loss: bool = True) -> dict:
    """PPO mini-batch -> TPR forest schedule -> one gradient finalisation."""
    if forward_only:
        raise NotImplementedError("the TPR PPO schedule is training-only")
    import os

    from ..utils.capture import ENV_DIR, capture_actor_update_minibatch

    if os.environ.get(ENV_DIR) and isinstance(data, dict):
        idx = getattr(engine, "_tpr_capture_count", 0)
        capture_actor_update_minibatch(data, batch_idx=idx, capture_index=idx)
        engine._tpr_capture_count = idx + 1
    return execute_prepared_tpr_batch(engine, prepare_tpr_batch(engine, data, loss_function), sync_loss=sync_loss)
