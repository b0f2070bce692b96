"""Absolute RoPE positions for a segment, in a shard's physical row order.

A segment that starts at absolute position ``P`` uses positions
``P + shard.physical_global_indices()``; padding rows repeat the last valid
position so they stay finite (they are masked out of attention anyway).  The
model's :class:`~bridge_b200.models.layers.RotaryEmbedding` turns positions into
cos/sin tables; RoPE itself is applied inside the fused qk-norm+RoPE kernel.

Parity: verl/models/mcore/tpr/rope.py:49-163 (build_suffix_rotary_pos_emb,
build_sharded_rotary_pos_emb, disable_bound_context_parallel_sharding).
"""

from __future__ import annotations

from contextlib import contextmanager

import torch
from torch import Tensor

from .shard import SequenceShard


def _check(name: str, value: int, *, zero_ok: bool) -> None:
    lo = 0 if zero_ok else 1
    if not isinstance(value, int) or isinstance(value, bool) or value < lo:
        raise ValueError(f"{name} must be a {'non-negative' if zero_ok else 'positive'} integer, got {value!r}")


def sharded_position_ids(position_start: int, shard: SequenceShard, *, device=None) -> Tensor:
    """Absolute position of every local physical row (padding -> last valid)."""
    _check("position_start", position_start, zero_ok=True)
    return shard.global_indices(device=device) + position_start


def build_suffix_rotary_pos_emb(rotary_embedding, *, prefix_length: int, suffix_length: int,
                                disable_context_parallel_sharding: bool = False) -> Tensor:
    """RoPE table (``[suffix, rotary_dim]`` cos|sin packed) for positions ``[P, P+b)``."""
    _check("prefix_length", prefix_length, zero_ok=True)
    _check("suffix_length", suffix_length, zero_ok=False)
    if not callable(rotary_embedding):
        raise TypeError("rotary_embedding must be callable")
    pos = torch.arange(prefix_length, prefix_length + suffix_length, dtype=torch.long)
    return rotary_embedding(pos)


def build_sharded_rotary_pos_emb(rotary_embedding, *, position_start: int, shard: SequenceShard,
                                 disable_context_parallel_sharding: bool = False) -> Tensor:
    """RoPE table for the shard's local rows, in physical order."""
    if not isinstance(shard, SequenceShard):
        raise TypeError(f"shard must implement SequenceShard, got {type(shard).__name__}")
    table = rotary_embedding(sharded_position_ids(position_start, shard))
    if table.shape[0] != shard.local_length:
        raise RuntimeError(f"sharded rotary embedding length must be {shard.local_length}, got {table.shape[0]}")
    return table


@contextmanager
def disable_bound_context_parallel_sharding(rotary_embedding):
    """Positions here are always explicit, so a bound CP slicer has nothing to undo."""
    if not hasattr(rotary_embedding, "cp_group"):
        yield
        return
    saved = rotary_embedding.cp_group
    rotary_embedding.cp_group = None
    try:
        yield
    finally:
        rotary_embedding.cp_group = saved
