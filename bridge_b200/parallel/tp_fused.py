"""Sequence-parallel TP linears whose collective is fused into the tcgen05 GEMM over NVLink.

* :func:`ag_linear` (column-parallel): ``y[M, N/tp] = all_gather(x[M/tp, K]) @ W^T`` in ONE kernel --
  the GEMM pulls the peers' token rows into a local buffer itself (P2P loads) while its first
  tiles run on the local rows.  Backward: ``dx`` = GEMM + reduce-scatter kernel, ``dW`` accumulates
  ``dy^T x_full`` into the FP32 main gradient.
* :func:`linear_rs` (row-parallel): ``y[M/tp, N] = reduce_scatter(x[M, K/tp] @ W^T)``: the GEMM epilogue
  stores each output row into its owner's receive slot (P2P stores); the owner sums the slots.
  Backward: ``dx`` = all-gather + GEMM kernel on ``dy``, ``dW`` from the gathered ``dy``.

Each call uses one of two symmetric workspaces (alternating) and exactly one cross-GPU barrier:
before the kernel for the all-gather (every rank's staging is written), after it for the
reduce-scatter (every slot has landed).  With two alternating buffers that one barrier also
guarantees no rank overwrites a buffer a peer is still reading from the call before.  Every TP
rank must make the same sequence of calls (true for SPMD model code).

Two implementations of the same pair of collectives (``TPR_TP_OVERLAP``):

* ``kernel`` -- the single-launch fused tcgen05 kernels described above;
* ``split`` (default) -- the CTA-pair tcgen05 GEMM (the fastest GEMM of this framework) on row blocks,
  with the NVLink traffic on a side stream under it, moved by the copy engines (``p2p_copy``: no SMs
  taken from the GEMM).  AG: the local rows' GEMM starts at once while the peers' rows are pulled; the
  remote rows' GEMM follows.  RS: the GEMMs of the peers' row blocks write into this rank's symmetric
  send slots first; after one barrier the side stream pulls the peers' slots for this rank's rows
  while the local block's GEMM runs; one add finishes.  Each call still uses one barrier; the side stream always rejoins the
  compute stream before the call returns, so the two-buffer argument above still holds.

Parity: Megatron sequence-parallel ColumnParallelLinear / RowParallelLinear as used by the
reference's TP2 path (verl/models/mcore/tpr/attention.py:117-126, 195-221).
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch import Tensor

from ..ops._ext import kernels
from ..ops.gemm import gemm

_MODE = os.environ.get("TPR_TP_COMM", "auto")  # auto | nvlink | nccl
_OVERLAP = os.environ.get("TPR_TP_OVERLAP", "split")  # split | kernel
_COMMS: dict = {}


def set_tp_comm_mode(mode: str) -> None:
    global _MODE
    if mode not in ("auto", "nvlink", "nccl"):
        raise ValueError(f"unknown tp_comm mode {mode!r}")
    _MODE = mode


class TPFusedComm:
    def __init__(self, group, device: torch.device, capacity_bytes: int = 64 << 20,
                 timeout_s: float | None = None) -> None:
        from .symmetric import SymmetricHeap

        self.group = group
        self.heap = SymmetricHeap(group, device, timeout_s=timeout_s)
        self.n, self.rank = self.heap.size, self.heap.rank
        self.capacity = capacity_bytes
        self.timeout_s = self.heap.timeout_s
        self.bufs = [self.heap.alloc(capacity_bytes), self.heap.alloc(capacity_bytes)]
        self.calls = 0
        self.counters = torch.zeros(8192, dtype=torch.int32, device=device)

    def _next(self, nbytes: int):
        if nbytes > self.capacity:      # same shapes on every TP rank -> every rank grows together
            torch.cuda.synchronize()
            self.heap.barrier()
            self.capacity = max(nbytes, 2 * self.capacity)
            self.bufs = [self.heap.alloc(self.capacity), self.heap.alloc(self.capacity)]
        buf = self.bufs[self.calls % 2]
        self.calls += 1
        return buf

    def ag_gemm(self, x_local: Tensor, w: Tensor, *, b_mn: bool) -> tuple[Tensor, Tensor]:
        """``(all_gather(x_local) @ op(w)^T, all_gather(x_local))``."""
        ms, k = x_local.shape
        buf = self._next(ms * k * 2)
        buf.view(torch.bfloat16, ms * k).view(ms, k).copy_(x_local)
        gather = torch.empty((ms * self.n, k), dtype=x_local.dtype, device=x_local.device)
        gather[self.rank * ms:(self.rank + 1) * ms].copy_(x_local)
        self.heap.barrier()
        y = kernels().tp_ag_gemm(gather, w, b_mn, buf.ptrs, self.rank, ms, self.counters, self.timeout_s)
        return y, gather

    def gemm_rs(self, a: Tensor, w: Tensor, *, b_mn: bool) -> Tensor:
        """``reduce_scatter(a @ op(w)^T)`` over token rows: this rank's ``[M/n, N]``."""
        m, _ = a.shape
        if m % self.n:
            raise ValueError("token count must divide by the TP size under sequence parallelism")
        ms = m // self.n
        nout = w.shape[1] if b_mn else w.shape[0]
        buf = self._next(self.n * ms * nout * 2)
        kernels().tp_gemm_rs(a, w, b_mn, buf.ptrs, self.rank, ms, self.timeout_s)
        self.heap.barrier()
        return kernels().tp_sum_slots(buf.view(torch.bfloat16), self.n, ms, nout)

    # ---------------------------------------------------------------- split variant
    def _side(self):
        if getattr(self, "_side_stream", None) is None:
            self._side_stream = torch.cuda.Stream(device=self.heap.device)
            self._idx: dict = {}
        return self._side_stream

    def _rows_index(self, ms: int, device):
        key = ("ag", ms)
        got = self._idx.get(key)
        if got is None:
            ranks = torch.arange(self.n, dtype=torch.int32).repeat_interleave(ms)
            rows = torch.arange(ms, dtype=torch.int32).repeat(self.n)
            own = torch.arange(ms, dtype=torch.int32)
            got = self._idx[key] = (ranks.to(device), rows.to(device), own.to(device))
        return got

    def ag_gemm_split(self, x_local: Tensor, w: Tensor, *, b_mn: bool) -> tuple[Tensor, Tensor]:
        ms, k = x_local.shape
        n, r = self.n, self.rank
        nout = w.shape[1] if b_mn else w.shape[0]
        buf = self._next(ms * k * 2)
        buf.view(torch.bfloat16, ms * k).view(ms, k).copy_(x_local)
        gather = torch.empty((ms * n, k), dtype=x_local.dtype, device=x_local.device)
        y = torch.empty((ms * n, nout), dtype=x_local.dtype, device=x_local.device)
        self.heap.barrier()                                   # every rank's staging is written
        side, main = self._side(), torch.cuda.current_stream()
        ranks, rows, _ = self._rows_index(ms, x_local.device)
        ev = torch.cuda.Event()
        ev.record(main)
        with torch.cuda.stream(side):
            side.wait_event(ev)
            m = kernels()
            for j in range(n):      # copy engine: the NVLink pull takes no SMs from the GEMM below
                m.p2p_copy(gather[j * ms:(j + 1) * ms], buf.ptrs[j], ms * k * 2)
        gemm(x_local, w, b_mn=b_mn, out=y[r * ms:(r + 1) * ms])          # local rows meanwhile
        main.wait_stream(side)
        for j in range(n):
            if j != r:
                gemm(gather[j * ms:(j + 1) * ms], w, b_mn=b_mn, out=y[j * ms:(j + 1) * ms])
        gather.record_stream(side)
        return y, gather

    def gemm_rs_split(self, a: Tensor, w: Tensor, *, b_mn: bool) -> Tensor:
        m, _ = a.shape
        n, r = self.n, self.rank
        if m % n:
            raise ValueError("token count must divide by the TP size under sequence parallelism")
        ms = m // n
        nout = w.shape[1] if b_mn else w.shape[0]
        slot = ms * nout
        buf = self._next(n * slot * 2)
        slots = buf.view(torch.bfloat16, n * slot).view(n, ms, nout)
        for d in range(1, n):                                   # peers' blocks first
            j = (r + d) % n
            gemm(a[j * ms:(j + 1) * ms], w, b_mn=b_mn, out=slots[j])
        self.heap.barrier()                                   # every rank's blocks for every owner landed
        side, main = self._side(), torch.cuda.current_stream()
        parts = torch.empty((n - 1, ms, nout), dtype=a.dtype, device=a.device)
        ev = torch.cuda.Event()
        ev.record(main)
        with torch.cuda.stream(side):
            side.wait_event(ev)
            m = kernels()
            for i, j in enumerate(q for q in range(n) if q != r):   # the peers' partials for my rows
                m.p2p_copy(parts[i], buf.ptrs[j] + r * slot * 2, slot * 2)
        own = gemm(a[r * ms:(r + 1) * ms], w, b_mn=b_mn)                  # local block meanwhile
        main.wait_stream(side)
        parts.record_stream(side)
        return own.add_(parts[0]) if n == 2 else own.add_(parts.float().sum(0).to(own.dtype))

    def close(self) -> None:
        self.heap.close()


def fused_comm(group, x: Tensor) -> TPFusedComm | None:
    """The fused comm object for ``group`` when the NVLink path applies to ``x``, else None."""
    if _MODE == "nccl" or group is None or not x.is_cuda or x.dtype != torch.bfloat16:
        return None
    n = dist.get_world_size(group)
    local = int(os.environ.get("LOCAL_WORLD_SIZE", dist.get_world_size()))
    if not (1 < n <= 8 and local >= dist.get_world_size()):
        if _MODE == "nvlink":
            raise ValueError("tp_comm='nvlink' needs a single-node TP group of 2..8 GPUs")
        return None
    key = id(group)
    if key not in _COMMS:
        _COMMS[key] = TPFusedComm(group, x.device)
    return _COMMS[key]


def close_all() -> None:
    for c in _COMMS.values():
        c.close()
    _COMMS.clear()


def _wgrad(w: Tensor, dy: Tensor, x: Tensor):
    main = getattr(w, "main_grad", None)
    if main is not None:
        gemm(dy, x, a_mn=True, b_mn=True, out=main, accumulate=True)
        return None
    return gemm(dy, x, a_mn=True, b_mn=True)


def _ag(comm, x, w, b_mn):
    return (comm.ag_gemm_split if _OVERLAP == "split" else comm.ag_gemm)(x, w, b_mn=b_mn)


def _rs(comm, a, w, b_mn):
    return (comm.gemm_rs_split if _OVERLAP == "split" else comm.gemm_rs)(a, w, b_mn=b_mn)


class _AGLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, comm):
        y, gather = _ag(comm, x.contiguous(), w, False)
        ctx.save_for_backward(gather, w)
        ctx.comm = comm
        return y

    @staticmethod
    def backward(ctx, dy):
        gather, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = _rs(ctx.comm, dy, w, True)                   # reduce_scatter(dy @ W)
        dw = _wgrad(w, dy, gather)
        return dx, dw, None


class _LinearRS(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, comm):
        x = x.contiguous()
        y = _rs(comm, x, w, False)
        ctx.save_for_backward(x, w)
        ctx.comm = comm
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dx, dy_full = _ag(ctx.comm, dy.contiguous(), w, True)          # all_gather(dy) @ W
        dw = _wgrad(w, dy_full, x)
        return dx, dw, None


def ag_linear(x: Tensor, w: Tensor, comm: TPFusedComm) -> Tensor:
    return _AGLinear.apply(x, w, comm)


def linear_rs(x: Tensor, w: Tensor, comm: TPFusedComm) -> Tensor:
    return _LinearRS.apply(x, w, comm)
