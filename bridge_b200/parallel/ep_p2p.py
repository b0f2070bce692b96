"""Expert-parallel MoE dispatch / combine over NVLink peer memory.

Every rank publishes its expert-sorted token rows in a symmetric staging buffer; after one
cross-GPU barrier the owner of each expert pulls exactly the rows routed to its experts with P2P
loads (one warp per row), already grouped by local expert (expert-major, source rank minor), so
the grouped expert GEMM consumes them without a re-sort.  Combine is the mirror image: owners
publish expert outputs and every rank pulls its own rows back in its original sorted order.
Backward of dispatch is the combine gather of the gradients and vice versa (each row travels to
exactly one owner, so no reduction is needed).

The routing table (tokens per (source rank, expert)) is all-gathered once per layer call (one
small NCCL collective + a host read, as the NCCL all-to-all path also needs).  Each staging use is
write -> barrier -> peer reads with two alternating buffers (one barrier per use suffices).

Parity: replaces the NCCL all-to-all dispatch / combine of the MoE layer (the reference rejects
MoE; this is the build target "MoE dispatch/combine over peer memory").
"""

from __future__ import annotations

import os

import numpy as np
import torch
import torch.distributed as dist
from torch import Tensor

from ..ops._ext import kernels

_MODE = os.environ.get("TPR_EP_COMM", "auto")  # auto | nvlink | nccl
_COMMS: dict = {}


def set_ep_comm_mode(mode: str) -> None:
    global _MODE
    if mode not in ("auto", "nvlink", "nccl"):
        raise ValueError(f"unknown ep_comm mode {mode!r}")
    _MODE = mode


class EPP2PComm:
    def __init__(self, group, device: torch.device, capacity_bytes: int = 32 << 20):
        from .symmetric import SymmetricHeap

        self.group = group
        self.heap = SymmetricHeap(group, device)
        self.n, self.rank = self.heap.size, self.heap.rank
        self.device = device
        self.capacity = capacity_bytes
        self.bufs = [self.heap.alloc(capacity_bytes), self.heap.alloc(capacity_bytes)]
        self.uses = 0

    def next_buffer(self, nbytes: int):
        if nbytes > self.capacity:       # every EP rank takes the same decision (sizes all-gathered)
            torch.cuda.synchronize()
            self.heap.barrier()
            self.capacity = max(nbytes, 2 * self.capacity)
            self.bufs = [self.heap.alloc(self.capacity), self.heap.alloc(self.capacity)]
        buf = self.bufs[self.uses % 2]
        self.uses += 1
        return buf

    def publish_and_gather(self, rows: Tensor, src_rank: Tensor, src_row: Tensor, out_rows: int,
                           stage_rows: int) -> Tensor:
        """Write ``rows`` to my staging, barrier, pull ``out[i] = peer[src_rank[i]].staging[src_row[i]]``."""
        width = rows.shape[1]
        buf = self.next_buffer(max(stage_rows, 1) * width * 2)
        if rows.shape[0]:
            buf.view(torch.bfloat16, rows.shape[0] * width).view(rows.shape[0], width).copy_(rows)
        self.heap.barrier()
        out = torch.empty((out_rows, width), dtype=torch.bfloat16, device=rows.device)
        if out_rows:
            kernels().p2p_gather_rows(out, buf.ptrs, src_rank, src_row)
        return out

    def close(self) -> None:
        self.heap.close()


def ep_comm(group, x: Tensor) -> EPP2PComm | None:
    if _MODE == "nccl" or group is None or not x.is_cuda or x.dtype != torch.bfloat16:
        return None
    n = dist.get_world_size(group)
    local = int(os.environ.get("LOCAL_WORLD_SIZE", dist.get_world_size()))
    if not (1 < n <= 8 and local >= dist.get_world_size()) or (x.shape[1] * 2) % 16:
        if _MODE == "nvlink":
            raise ValueError("ep_comm='nvlink' needs a single-node EP group of 2..8 GPUs")
        return None
    key = id(group)
    if key not in _COMMS:
        _COMMS[key] = EPP2PComm(group, x.device)
    return _COMMS[key]


def close_all() -> None:
    for c in _COMMS.values():
        c.close()
    _COMMS.clear()


def exchange_plan(table: np.ndarray, me: int, local_experts: int, device) -> dict:
    """Index maps from the all-gathered routing table ``table[source rank, expert]`` (host ints)."""
    n, E = table.shape
    src_off = np.zeros_like(table)
    src_off[:, 1:] = np.cumsum(table, axis=1)[:, :-1]           # row of expert e in source i's sorted rows
    # receive layout of every owner j: for e in j's experts, for i in ranks -> consecutive rows
    recv_off = np.zeros_like(table)
    recv_total = np.zeros(n, dtype=np.int64)
    for j in range(n):
        pos = 0
        for e in range(j * local_experts, (j + 1) * local_experts):
            for i in range(n):
                recv_off[i, e] = pos
                pos += table[i, e]
        recv_total[j] = pos
    mine = range(me * local_experts, (me + 1) * local_experts)
    d_rank, d_row = [], []
    for e in mine:
        for i in range(n):
            c = int(table[i, e])
            if c:
                d_rank.append(np.full(c, i, dtype=np.int32))
                d_row.append(np.arange(src_off[i, e], src_off[i, e] + c, dtype=np.int32))
    c_rank, c_row = [], []
    for e in range(E):
        c = int(table[me, e])
        if c:
            j = e // local_experts
            c_rank.append(np.full(c, j, dtype=np.int32))
            c_row.append(np.arange(recv_off[me, e], recv_off[me, e] + c, dtype=np.int32))

    def dev(parts):
        a = np.concatenate(parts) if parts else np.zeros(0, dtype=np.int32)
        return torch.from_numpy(a).to(device, non_blocking=True)

    counts_local = table[:, me * local_experts:(me + 1) * local_experts].sum(0)
    return {"d_rank": dev(d_rank), "d_row": dev(d_row), "c_rank": dev(c_rank), "c_row": dev(c_row),
            "recv_rows": int(recv_total[me]), "send_rows": int(table[me].sum()),
            "max_recv": int(recv_total.max()), "max_send": int(table.sum(1).max()),
            "counts_local": torch.from_numpy(counts_local.astype(np.int64)).to(device, non_blocking=True)}


class _Dispatch(torch.autograd.Function):
    @staticmethod
    def forward(ctx, xs, comm, plan):
        ctx.comm, ctx.plan = comm, plan
        return comm.publish_and_gather(xs.contiguous(), plan["d_rank"], plan["d_row"], plan["recv_rows"],
                                       plan["max_send"])

    @staticmethod
    def backward(ctx, g):
        p = ctx.plan
        return ctx.comm.publish_and_gather(g.contiguous(), p["c_rank"], p["c_row"], p["send_rows"],
                                           p["max_recv"]), None, None


class _Combine(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y_recv, comm, plan):
        ctx.comm, ctx.plan = comm, plan
        return comm.publish_and_gather(y_recv.contiguous(), plan["c_rank"], plan["c_row"], plan["send_rows"],
                                       plan["max_recv"])

    @staticmethod
    def backward(ctx, g):
        p = ctx.plan
        return ctx.comm.publish_and_gather(g.contiguous(), p["d_rank"], p["d_row"], p["recv_rows"],
                                           p["max_send"]), None, None


def ep_moe_experts(xs: Tensor, counts_all: Tensor, comm: EPP2PComm, local_experts: int, experts_fn) -> Tensor:
    """``xs`` expert-sorted rows of this rank, ``counts_all [E]`` (device) -> expert outputs in ``xs`` order."""
    table_t = torch.empty((comm.n, counts_all.numel()), dtype=counts_all.dtype, device=counts_all.device)
    dist.all_gather_into_tensor(table_t, counts_all.contiguous(), group=comm.group)
    table = table_t.cpu().numpy().astype(np.int64)
    plan = exchange_plan(table, comm.rank, local_experts, xs.device)
    x_recv = _Dispatch.apply(xs, comm, plan)
    y_recv = experts_fn(x_recv, plan["counts_local"])
    return _Combine.apply(y_recv, comm, plan)
