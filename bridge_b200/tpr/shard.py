"""Ownership of one segment's token positions by one context-parallel rank.

Every shard is an ordered list of disjoint global ranges inside
``[0, padded_length)``.  Three concrete shapes exist:

* :class:`PrefixShard` -- one contiguous equal slice per rank (all-gather /
  Ulysses backends, and the CP=1 "full" shard);
* :class:`RangeSequenceShard` -- several ranges per rank (ring zigzag, hybrid);
* :class:`PaddedSequenceShard` -- wraps a physical shard of a length padded up
  to the backend's alignment, while loss/topology queries stay restricted to
  the logical ``[0, logical_length)``.  Padding rows reuse the last valid
  position id and are masked out of attention.

Zigzag layout (ring): the padded length is cut into ``2*cp`` chunks and rank r
owns chunks ``r`` and ``2*cp-1-r`` so causal work is balanced.

Parity: verl/models/mcore/tpr/shard.py:57-449 (protocol and the three shard
types), parallel/ring_attention.py:119-154 (zigzag), parallel/hybrid_attention.py:206-255
(hybrid = ring zigzag split into contiguous Ulysses pieces).
"""

from __future__ import annotations

from dataclasses import dataclass
from math import gcd
from typing import Protocol, runtime_checkable

import torch
from torch import Tensor

SequenceRange = tuple[int, int]


def _int_at_least(name: str, value, minimum: int) -> int:
    if not isinstance(value, int) or isinstance(value, bool) or value < minimum:
        raise ValueError(f"{name} must be an integer >= {minimum}, got {value!r}")
    return value


def _check_coords(cp_rank: int, cp_size: int) -> None:
    _int_at_least("cp_size", cp_size, 1)
    _int_at_least("cp_rank", cp_rank, 0)
    if cp_rank >= cp_size:
        raise ValueError(f"cp_rank must be in [0, {cp_size}), got {cp_rank}")


def _seq_dim(tensor: Tensor, dim: int) -> int:
    if tensor.ndim == 0:
        raise ValueError("tensor must have a sequence dimension")
    if not -tensor.ndim <= dim < tensor.ndim:
        raise ValueError(f"dim {dim} out of range for a {tensor.ndim}-D tensor")
    return dim % tensor.ndim


def _check_offset(offset: int, length: int) -> None:
    _int_at_least("global_offset", offset, 0)
    if offset >= length:
        raise ValueError(f"global_offset must be in [0, {length}), got {offset}")


@runtime_checkable
class SequenceShard(Protocol):
    @property
    def global_length(self) -> int: ...
    @property
    def padded_length(self) -> int: ...
    @property
    def local_length(self) -> int: ...
    @property
    def valid_local_length(self) -> int: ...
    @property
    def cp_rank(self) -> int: ...
    @property
    def cp_size(self) -> int: ...
    @property
    def global_ranges(self) -> tuple[SequenceRange, ...]: ...
    @property
    def physical_global_ranges(self) -> tuple[SequenceRange, ...]: ...
    @property
    def is_full(self) -> bool: ...
    def select(self, tensor: Tensor, *, dim: int = 0) -> Tensor: ...
    def global_indices(self, *, device=None) -> Tensor: ...
    def physical_global_indices(self, *, device=None) -> Tensor: ...
    def owns(self, global_offset: int) -> bool: ...
    def global_to_local(self, global_offset: int) -> int | None: ...
    def local_to_global(self, local_offset: int) -> int: ...


class _RangeOps:
    """Shared range arithmetic for shards whose ranges cover ``global_length``."""

    __slots__ = ()

    def _ranges(self) -> tuple[SequenceRange, ...]:  # pragma: no cover - overridden
        raise NotImplementedError

    @property
    def local_length(self) -> int:
        return sum(e - s for s, e in self._ranges())

    @property
    def padded_length(self) -> int:
        return self.global_length

    @property
    def valid_local_length(self) -> int:
        return self.local_length

    @property
    def global_ranges(self) -> tuple[SequenceRange, ...]:
        return self._ranges()

    @property
    def physical_global_ranges(self) -> tuple[SequenceRange, ...]:
        return self._ranges()

    def select(self, tensor: Tensor, *, dim: int = 0) -> Tensor:
        dim = _seq_dim(tensor, dim)
        if tensor.shape[dim] != self.global_length:
            raise ValueError(f"tensor sequence dimension must be {self.global_length}, got {tensor.shape[dim]}")
        parts = [tensor.narrow(dim, s, e - s) for s, e in self._ranges()]
        return parts[0] if len(parts) == 1 else torch.cat(parts, dim=dim)

    def global_indices(self, *, device=None) -> Tensor:
        parts = [torch.arange(s, e, dtype=torch.long, device=device) for s, e in self._ranges()]
        return parts[0] if len(parts) == 1 else torch.cat(parts)

    def physical_global_indices(self, *, device=None) -> Tensor:
        return self.global_indices(device=device)

    def owns(self, global_offset: int) -> bool:
        _check_offset(global_offset, self.global_length)
        return any(s <= global_offset < e for s, e in self._ranges())

    def global_to_local(self, global_offset: int) -> int | None:
        _check_offset(global_offset, self.global_length)
        base = 0
        for s, e in self._ranges():
            if s <= global_offset < e:
                return base + global_offset - s
            base += e - s
        return None

    def local_to_global(self, local_offset: int) -> int:
        _int_at_least("local_offset", local_offset, 0)
        if local_offset >= self.local_length:
            raise ValueError(f"local_offset must be in [0, {self.local_length}), got {local_offset}")
        rest = local_offset
        for s, e in self._ranges():
            if rest < e - s:
                return s + rest
            rest -= e - s
        raise AssertionError("unreachable")


@dataclass(frozen=True, slots=True)
class PrefixShard(_RangeOps):
    """Contiguous equal slice ``[rank*L/cp, (rank+1)*L/cp)``."""

    global_length: int
    local_start: int
    local_end: int
    cp_rank: int = 0
    cp_size: int = 1

    def __post_init__(self) -> None:
        _int_at_least("global_length", self.global_length, 1)
        _int_at_least("local_start", self.local_start, 0)
        _int_at_least("local_end", self.local_end, 0)
        _check_coords(self.cp_rank, self.cp_size)
        if self.global_length % self.cp_size:
            raise ValueError(f"global_length {self.global_length} must be divisible by cp_size {self.cp_size}")
        n = self.global_length // self.cp_size
        want = (self.cp_rank * n, (self.cp_rank + 1) * n)
        if (self.local_start, self.local_end) != want:
            raise ValueError(
                f"contiguous shard range mismatch: rank {self.cp_rank}/{self.cp_size} must own "
                f"[{want[0]}, {want[1]}), got [{self.local_start}, {self.local_end})"
            )

    @classmethod
    def full(cls, global_length: int) -> "PrefixShard":
        return cls(global_length, 0, global_length)

    @classmethod
    def contiguous(cls, global_length: int, *, cp_rank: int, cp_size: int) -> "PrefixShard":
        _int_at_least("global_length", global_length, 1)
        _check_coords(cp_rank, cp_size)
        if global_length % cp_size:
            raise ValueError(f"global_length {global_length} must be divisible by cp_size {cp_size}")
        n = global_length // cp_size
        return cls(global_length, cp_rank * n, (cp_rank + 1) * n, cp_rank=cp_rank, cp_size=cp_size)

    def _ranges(self):
        return ((self.local_start, self.local_end),)

    @property
    def is_full(self) -> bool:
        return self.cp_size == 1


@dataclass(frozen=True, slots=True)
class RangeSequenceShard(_RangeOps):
    """Ordered, disjoint, non-empty global ranges owned by one rank."""

    global_length: int
    ranges: tuple[SequenceRange, ...]
    cp_rank: int
    cp_size: int

    def __post_init__(self) -> None:
        _int_at_least("global_length", self.global_length, 1)
        _check_coords(self.cp_rank, self.cp_size)
        norm = tuple(tuple(r) for r in self.ranges)
        if not norm:
            raise ValueError("ranges must contain at least one non-empty range")
        prev = 0
        for i, r in enumerate(norm):
            if len(r) != 2:
                raise ValueError(f"ranges[{i}] must be a (start, end) pair, got {r!r}")
            s, e = r
            _int_at_least(f"ranges[{i}].start", s, 0)
            _int_at_least(f"ranges[{i}].end", e, 1)
            if s >= e:
                raise ValueError(f"ranges[{i}] must be non-empty, got [{s}, {e})")
            if e > self.global_length:
                raise ValueError(f"ranges[{i}] ends at {e}, beyond global_length {self.global_length}")
            if i and s < prev:
                raise ValueError("ranges must be ordered and non-overlapping")
            prev = e
        object.__setattr__(self, "ranges", norm)

    def _ranges(self):
        return self.ranges

    @property
    def is_full(self) -> bool:
        return self.ranges == ((0, self.global_length),)


@dataclass(frozen=True, slots=True)
class PaddedSequenceShard:
    """Logical segment of ``logical_length`` over a longer padded physical shard."""

    logical_length: int
    physical_shard: PrefixShard | RangeSequenceShard

    def __post_init__(self) -> None:
        _int_at_least("logical_length", self.logical_length, 1)
        if not isinstance(self.physical_shard, (PrefixShard, RangeSequenceShard)):
            raise TypeError(
                f"physical_shard must be PrefixShard or RangeSequenceShard, got {type(self.physical_shard).__name__}"
            )
        if self.logical_length >= self.physical_shard.global_length:
            raise ValueError(
                "PaddedSequenceShard requires logical_length smaller than the physical length, got "
                f"{self.logical_length} and {self.physical_shard.global_length}"
            )

    @property
    def global_length(self) -> int:
        return self.logical_length

    @property
    def padded_length(self) -> int:
        return self.physical_shard.global_length

    @property
    def local_length(self) -> int:
        return self.physical_shard.local_length

    @property
    def valid_local_length(self) -> int:
        return sum(e - s for s, e in self.global_ranges)

    @property
    def cp_rank(self) -> int:
        return self.physical_shard.cp_rank

    @property
    def cp_size(self) -> int:
        return self.physical_shard.cp_size

    @property
    def physical_global_ranges(self) -> tuple[SequenceRange, ...]:
        return self.physical_shard.global_ranges

    @property
    def global_ranges(self) -> tuple[SequenceRange, ...]:
        n = self.logical_length
        return tuple((s, min(e, n)) for s, e in self.physical_global_ranges if s < n)

    @property
    def is_full(self) -> bool:
        return self.cp_size == 1 and self.valid_local_length == self.logical_length

    def select(self, tensor: Tensor, *, dim: int = 0) -> Tensor:
        dim = _seq_dim(tensor, dim)
        if tensor.shape[dim] != self.logical_length:
            raise ValueError(f"tensor sequence dimension must be {self.logical_length}, got {tensor.shape[dim]}")
        pad = list(tensor.shape)
        pad[dim] = self.padded_length - self.logical_length
        return self.physical_shard.select(torch.cat((tensor, tensor.new_zeros(pad)), dim=dim), dim=dim)

    def global_indices(self, *, device=None) -> Tensor:
        return self.physical_global_indices(device=device).clamp_max(self.logical_length - 1)

    def physical_global_indices(self, *, device=None) -> Tensor:
        return self.physical_shard.global_indices(device=device)

    def owns(self, global_offset: int) -> bool:
        _check_offset(global_offset, self.logical_length)
        return self.physical_shard.owns(global_offset)

    def global_to_local(self, global_offset: int) -> int | None:
        _check_offset(global_offset, self.logical_length)
        return self.physical_shard.global_to_local(global_offset)

    def local_to_global(self, local_offset: int) -> int:
        g = self.physical_shard.local_to_global(local_offset)
        if g >= self.logical_length:
            raise ValueError(f"local offset {local_offset} refers to a padding token")
        return g

    def valid_mask(self, *, device=None) -> Tensor:
        """Bool per local row: True where the row is a real (non-padding) token."""
        return self.physical_global_indices(device=device) < self.logical_length


def round_up_sequence_length(logical_length: int, alignment: int) -> int:
    _int_at_least("logical_length", logical_length, 1)
    _int_at_least("alignment", alignment, 1)
    return -(-logical_length // alignment) * alignment


def maybe_pad_sequence_shard(logical_length: int, physical_shard) -> SequenceShard:
    if logical_length == physical_shard.global_length:
        return physical_shard
    return PaddedSequenceShard(logical_length, physical_shard)


def physical_sequence_shard(shard: SequenceShard):
    return shard.physical_shard if isinstance(shard, PaddedSequenceShard) else shard


def iter_valid_sequence_slices(shard: SequenceShard) -> tuple[tuple[SequenceRange, slice], ...]:
    """``((global_start, global_end), local_slice)`` for every non-empty logical range."""
    out = []
    base = 0
    for s, e in shard.physical_global_ranges:
        end = min(e, shard.global_length)
        if s < end:
            out.append(((s, end), slice(base, base + end - s)))
        base += e - s
    if sum(r[1] - r[0] for r, _ in out) != shard.valid_local_length:
        raise RuntimeError("valid sequence slices do not match shard validity metadata")
    return tuple(out)


def local_valid_mask(shard: SequenceShard, *, device=None) -> Tensor:
    """Bool ``[local_length]``: True for real tokens, False for padding rows."""
    return shard.physical_global_indices(device=device) < shard.global_length


# --------------------------------------------------------------------------- zigzag / hybrid
def make_ring_sequence_shard(global_length: int, *, cp_rank: int, cp_size: int) -> SequenceShard:
    """Zigzag shard: rank r owns chunks ``r`` and ``2*cp-1-r`` of ``2*cp`` equal chunks."""
    _int_at_least("global_length", global_length, 1)
    _check_coords(cp_rank, cp_size)
    padded = round_up_sequence_length(global_length, 2 * cp_size)
    c = padded // (2 * cp_size)
    lo, hi = cp_rank, 2 * cp_size - 1 - cp_rank
    phys = RangeSequenceShard(padded, ((lo * c, (lo + 1) * c), (hi * c, (hi + 1) * c)), cp_rank, cp_size)
    return maybe_pad_sequence_shard(global_length, phys)


def hybrid_alignment(cp_size: int, ulysses_size: int) -> int:
    ring = cp_size // ulysses_size
    a, b = cp_size, 2 * ring
    return a * b // gcd(a, b)


def make_hybrid_sequence_shard(global_length: int, *, cp_rank: int, cp_size: int,
                               ulysses_size: int) -> SequenceShard:
    """Ring zigzag over ``R = cp/U`` ring ranks, each zigzag shard split in U pieces.

    ``cp_rank = ring_rank * U + ulysses_rank``; piece ``ulysses_rank`` of the
    ring rank's (concatenated) zigzag shard is owned by this rank.
    """
    _int_at_least("global_length", global_length, 1)
    _check_coords(cp_rank, cp_size)
    _int_at_least("ulysses_size", ulysses_size, 1)
    if cp_size % ulysses_size:
        raise ValueError(f"cp_size {cp_size} must be divisible by ulysses_size {ulysses_size}")
    ring = cp_size // ulysses_size
    ring_rank, u_rank = divmod(cp_rank, ulysses_size)
    padded = round_up_sequence_length(global_length, hybrid_alignment(cp_size, ulysses_size))
    c = padded // (2 * ring)
    ring_ranges = ((ring_rank * c, (ring_rank + 1) * c),
                   ((2 * ring - 1 - ring_rank) * c, (2 * ring - ring_rank) * c))
    piece = 2 * c // ulysses_size
    lo, hi = u_rank * piece, (u_rank + 1) * piece
    ranges: list[SequenceRange] = []
    base = 0
    for s, e in ring_ranges:
        a, b = max(lo, base), min(hi, base + e - s)
        if a < b:
            ranges.append((s + a - base, s + b - base))
        base += e - s
    merged: list[SequenceRange] = []
    for s, e in ranges:
        if merged and merged[-1][1] == s:
            merged[-1] = (merged[-1][0], e)
        else:
            merged.append((s, e))
    phys = RangeSequenceShard(padded, tuple(merged), cp_rank, cp_size)
    return maybe_pad_sequence_shard(global_length, phys)
