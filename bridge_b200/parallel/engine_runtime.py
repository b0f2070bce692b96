"""Engine-level context-parallel runtime: group, backend, CP loss aggregation.

The backend name comes from ``engine_config.tpr_cp_backend``, else from
``context_parallel_algo`` (engine config, then the model config); with CP > 1
and nothing configured the default is ``allgather``.

Parity: verl/models/mcore/tpr/parallel/engine_runtime.py:31-145.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor

from .backend import ALLGATHER_CP_BACKEND, resolve_tpr_cp_backend


@dataclass(frozen=True)
class TPREngineCPRuntime:
    group: Any
    size: int
    rank: int
    backend: Any

    @property
    def enabled(self) -> bool:
        return self.group is not None


def configured_cp_algorithm(engine) -> str | None:
    ec = getattr(engine, "engine_config", None)
    for source in (getattr(ec, "tpr_cp_backend", None), getattr(ec, "context_parallel_algo", None),
                   getattr(getattr(engine, "model_config", None), "context_parallel_algo", None)):
        if source:
            return str(source)
    return None


def resolve_engine_cp_runtime(engine) -> TPREngineCPRuntime:
    ps = engine.parallel
    if ps.cp == 1 or ps.cp_group is None:
        return TPREngineCPRuntime(None, 1, 0, None)
    name = configured_cp_algorithm(engine) or ALLGATHER_CP_BACKEND
    backend = resolve_tpr_cp_backend(name, cp_group=ps.cp_group, parallel_size=ps.cp, parallel_rank=ps.cp_rank)
    return TPREngineCPRuntime(ps.cp_group, ps.cp, ps.cp_rank, backend)


def aggregate_cp_loss(loss_sum: Tensor, normalized_loss: Tensor, runtime: TPREngineCPRuntime):
    """Sum per-rank loss contributions over the CP group (two scalars, one collective)."""
    if runtime.group is None:
        return loss_sum, normalized_loss
    both = torch.stack([loss_sum.detach().float(), normalized_loss.detach().float()])
    dist.all_reduce(both, group=runtime.group)
    return both[0], both[1]
