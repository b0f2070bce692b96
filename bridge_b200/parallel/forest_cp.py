"""Segment-granular context parallelism for the batched forest executor.

The forest executor forwards a packed chunk of many segments at a time.  Under context parallelism
the chunk's segments are *partitioned* over the CP group -- a contiguous minimax split by token
count, so siblings stay together and every rank carries the same number of tokens (up to one
segment) -- and each rank forwards only its own segments.  A segment's own causal attention, its
GDN recurrence and its loss rows then need no data from another rank: per layer there is no
attention collective at all.  What crosses ranks is what descendants on other ranks read:

* after a chunk of internal segments is pushed, every attention layer's new K/V rows and every GDN
  layer's final (conv, recurrent) state are all-gathered once into a replicated *anchor bank*
  (rank-major row order), which the children of those segments address through prefix spans;
* backward: each rank's anchor gradient (from its own descendants' queries) is summed into the
  rows' owner (reduce to owner, fixed rank order, FP32 accumulation) and flows into the owner's
  local K/V graph.

Compared with splitting every segment over the ranks (the per-segment CP backends), this keeps the
attention and GEMM tiles full (whole 512-token segments instead of 64-row zigzag pieces) and moves
one K/V copy per pushed segment instead of one per layer per forward.  Segments longer than a
rank's token budget cannot be placed whole; the engine runs those forests through the per-segment
CP backends instead.

Transport: on a single-node CUDA group the rows move by NVLink P2P (symmetric staging buffer, one
cross-GPU barrier, ``p2p_gather_rows`` pulls / ``p2p_reduce_rows`` owner sums); elsewhere (and as
the baseline) by ``all_gather`` + ``all_reduce`` of the process group (NCCL or gloo).

Parity: the prefix-KV relay of verl/models/mcore/tpr/parallel/execution_context.py:166-180 and
kv_stack.py:175-203 (ancestor K/V visible to every descendant, dK/dV accumulated back to the
producer); the placement and transport are this framework's own.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor


def partition_contiguous(costs: list[int], parts: int) -> list[tuple[int, int]]:
    """Split ``costs`` into ``parts`` contiguous ranges minimising the largest range sum.

    Binary search on the bound with a greedy fill; ranges may be empty when there are fewer items
    than parts (the trailing ranks get nothing).
    """
    n = len(costs)
    if parts <= 0:
        raise ValueError("parts must be positive")
    if n == 0:
        return [(0, 0)] * parts

    def fill(bound: int) -> list[tuple[int, int]] | None:
        out, s, acc = [], 0, 0
        for i, c in enumerate(costs):
            if c > bound:
                return None
            if acc + c > bound:
                out.append((s, i))
                s, acc = i, 0
            acc += c
        out.append((s, n))
        return out if len(out) <= parts else None

    lo, hi = max(costs), sum(costs)
    while lo < hi:
        mid = (lo + hi) // 2
        if fill(mid) is None:
            lo = mid + 1
        else:
            hi = mid
    ranges = fill(lo)
    assert ranges is not None
    # Spread: split the largest multi-item ranges while ranks are left over (more ranks busy,
    # same bound), then pad with empty ranges.
    while len(ranges) < parts:
        best = max(range(len(ranges)), key=lambda j: (ranges[j][1] - ranges[j][0] > 1,
                                                      sum(costs[ranges[j][0]:ranges[j][1]])))
        s, e = ranges[best]
        if e - s <= 1:
            break
        tot, acc, cut = sum(costs[s:e]), 0, s + 1
        for i in range(s, e - 1):
            acc += costs[i]
            cut = i + 1
            if 2 * acc >= tot:
                break
        ranges[best:best + 1] = [(s, cut), (cut, e)]
    while len(ranges) < parts:
        ranges.append((n, n))
    return ranges


class ForestCP:
    """CP group handle of the forest executor: segment placement + anchor row exchange."""

    def __init__(self, group, *, comm: str = "auto") -> None:
        if comm not in ("auto", "nvlink", "nccl"):
            raise ValueError(f"unknown CP comm mode {comm!r}")
        self.group = group
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.comm_mode = comm
        self._p2p = None
        self._index_cache: dict = {}

    # ------------------------------------------------------------------ placement
    def split(self, nodes: list) -> list[list]:
        """Per-rank node lists (contiguous minimax partition by token count)."""
        ranges = partition_contiguous([n.length for n in nodes], self.size)
        return [nodes[s:e] for s, e in ranges]

    # ------------------------------------------------------------------ transport selection
    def _p2p_comm(self, like: Tensor):
        if self.comm_mode == "nccl" or not like.is_cuda:
            return None
        if self._p2p is None:
            import os

            local = int(os.environ.get("LOCAL_WORLD_SIZE", dist.get_world_size()))
            ok = 1 < self.size <= 8 and local >= dist.get_world_size()
            if not ok:
                if self.comm_mode == "nvlink":
                    raise ValueError("cp_comm='nvlink' needs a single-node CP group of 2..8 GPUs")
                self.comm_mode = "nccl"
                return None
            from .cp_p2p import shared_cp_comm

            self._p2p = shared_cp_comm(self.group, like.device)
        return self._p2p

    def _indices(self, counts: tuple[int, ...], device):
        key = (counts, str(device))
        got = self._index_cache.get(key)
        if got is None:
            ranks = torch.repeat_interleave(torch.arange(self.size, dtype=torch.int32),
                                            torch.tensor(counts, dtype=torch.int64))
            rows = torch.cat([torch.arange(c, dtype=torch.int32) for c in counts])
            start = sum(counts[:self.rank])
            own = torch.arange(start, start + counts[self.rank], dtype=torch.int32)
            got = (ranks.to(device), rows.to(device), own.to(device))
            self._index_cache[key] = got
        return got

    # ------------------------------------------------------------------ gather / reduce
    def gather(self, tensors: list[Tensor], counts: list[int]) -> list[Tensor]:
        """All-gather dim-0 rows: rank ``j`` contributes ``counts[j]`` rows of every tensor; the result
        holds all ranks' rows in rank order.  Differentiable: the backward sums the gradient of each
        row over the ranks into its owner."""
        counts = tuple(int(c) for c in counts)
        if len(counts) != self.size:
            raise ValueError("one row count per CP rank is required")
        for t in tensors:
            if t.shape[0] != counts[self.rank]:
                raise ValueError(f"local tensor has {t.shape[0]} rows, expected {counts[self.rank]}")
        return list(_GatherRowsFn.apply(self, counts, *tensors))

    @staticmethod
    def _layout(shapes_bytes: list[int], rows: int) -> tuple[list[int], int]:
        offs, off = [], 0
        for rb in shapes_bytes:
            offs.append(off)
            off += (rows * rb + 255) // 256 * 256
        return offs, max(off, 256)

    def _all_gather_rows(self, local: list[Tensor], counts: tuple[int, ...]) -> list[Tensor]:
        total, mx = sum(counts), max(counts)
        p2p = self._p2p_comm(local[0]) if local else None
        outs = [t.new_empty((total, *t.shape[1:])) for t in local]
        if p2p is not None:
            widths = [max(1, t.numel() // max(t.shape[0], 1)) for t in outs]
            row_bytes = [w * t.element_size() for w, t in zip(widths, outs)]
            offs, nbytes = self._layout(row_bytes, mx)
            buf = p2p.next_buffer(nbytes)
            for t, o, rb in zip(local, offs, row_bytes):
                if t.shape[0]:
                    buf.local[o:o + t.shape[0] * rb].view(t.dtype).view(t.shape).copy_(t)
            p2p.heap.barrier()
            ranks, rows, _ = self._indices(counts, local[0].device)
            m = _kernels()
            for out, o, rb, w in zip(outs, offs, row_bytes, widths):
                if total:
                    m.p2p_gather_rows(out.view(total, w), [p + o for p in buf.ptrs], ranks, rows)
            return outs
        for t, out in zip(local, outs):
            pad = t.new_zeros((mx, *t.shape[1:]))
            pad[:t.shape[0]] = t
            parts = [torch.empty_like(pad) for _ in range(self.size)]
            dist.all_gather(parts, pad.contiguous(), group=self.group)
            torch.cat([p[:c] for p, c in zip(parts, counts)], out=out)
        return outs

    def _reduce_rows_to_owner(self, grads: list[Tensor], counts: tuple[int, ...]) -> list[Tensor]:
        total = sum(counts)
        me, start = counts[self.rank], sum(counts[:self.rank])
        p2p = self._p2p_comm(grads[0]) if grads else None
        if p2p is not None:
            widths = [max(1, g.numel() // max(g.shape[0], 1)) for g in grads]
            row_bytes = [w * g.element_size() for w, g in zip(widths, grads)]
            offs, nbytes = self._layout(row_bytes, total)
            buf = p2p.next_buffer(nbytes)
            for g, o, rb in zip(grads, offs, row_bytes):
                if total:
                    buf.local[o:o + total * rb].view(g.dtype).view(g.shape).copy_(g)
            p2p.heap.barrier()
            _, _, own = self._indices(counts, grads[0].device)
            m = _kernels()
            outs = []
            for g, o, w in zip(grads, offs, widths):
                out = g.new_empty((me, *g.shape[1:]))
                if me:
                    m.p2p_reduce_rows(out.view(me, w), [p + o for p in buf.ptrs], own, g.dtype == torch.float32, None)
                outs.append(out)
            return outs
        outs = []
        for g in grads:
            acc = g.float().contiguous() if g.dtype != torch.float32 else g.clone().contiguous()
            dist.all_reduce(acc, group=self.group)
            outs.append(acc[start:start + me].to(g.dtype))
        return outs


_STACK_CP: dict = {}


def gather_stack(x: Tensor, group) -> Tensor:
    """``[n, *x.shape]``: every CP rank's ``x`` (differentiable; the backward returns this rank's slice of
    the stacked gradient summed over ranks).  Moves over NVLink P2P on a single-node CUDA group (one
    staging write, one barrier, peer loads), else ``all_gather`` / ``all_reduce``."""
    cp = _STACK_CP.get(id(group))
    if cp is None:
        cp = _STACK_CP[id(group)] = ForestCP(group)
    row = x.reshape(1, -1)
    if (row.shape[1] * row.element_size()) % 16 and x.is_cuda:
        row = torch.nn.functional.pad(row, (0, (-row.shape[1]) % (16 // row.element_size())))
    out = cp.gather([row], [1] * cp.size)[0]
    return out[:, :x.numel()].reshape(cp.size, *x.shape)


def _kernels():
    from ..ops._ext import kernels

    return kernels()


class _GatherRowsFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, cp: ForestCP, counts, *local):
        ctx.cp, ctx.counts = cp, counts
        outs = cp._all_gather_rows([t.contiguous() for t in local], counts)
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        grads = [g.contiguous() for g in grads]
        locs = ctx.cp._reduce_rows_to_owner(grads, ctx.counts)
        return (None, None, *locs)
