"""Context-parallel attention over NVLink peer memory (B200 transport for the ring and all-gather backends).

Instead of CP-1 NCCL ring hops per block (or NCCL all-gathers), every rank publishes the local K/V
rows of all prefix blocks and of the current segment in a symmetric staging buffer; after one
cross-GPU barrier each rank pulls the rows it needs straight from its peers (P2P loads, one warp
per row) into a local bank laid out in global token order:

    bank = [prefix block 0 (valid rows) | prefix block 1 | ... | current segment (padded rows)]

Every contiguous range of local query rows ``[s, e)`` of the current segment is then one sequence
of the tcgen05 tree-attention kernel: causal over its own rows plus a prefix span ``bank[0, P + s)``
-- the zigzag ring's FULL / CAUSAL / SKIP block classes fall out of that structure without a mask.
Backward: the attention kernel produces d(bank); every rank publishes it and each owner pulls and
sums (fixed rank order, FP32) the gradient of its own rows from all peers -- the dK/dV of the ring's
travelling accumulator, returned over P2P.

Each use of the staging area is one write -> barrier -> peer reads; two alternating buffers make
that single barrier sufficient.  Shard layouts: contiguous (all-gather CP) and zigzag (ring CP).

Parity: the semantics of verl/models/mcore/tpr/parallel/ring_attention.py:57-1140 and
allgather_attention.py:55-382 (same shards, masks and gradients); the transport is new.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch import Tensor

from ..ops._ext import kernels
from ..tpr.shard import PrefixShard, RangeSequenceShard, physical_sequence_shard

_MODE = os.environ.get("TPR_CP_COMM", "auto")   # auto | nvlink | nccl
_COMMS: dict = {}


def set_cp_comm_mode(mode: str) -> None:
    global _MODE
    if mode not in ("auto", "nvlink", "nccl"):
        raise ValueError(f"unknown cp_comm mode {mode!r}")
    _MODE = mode


def rank_rows(shard, j: int) -> list[int]:
    """Global (padded) token indices of rank ``j``'s local rows for a contiguous or zigzag shard."""
    phys = physical_sequence_shard(shard)
    cp, padded = phys.cp_size, phys.global_length
    if isinstance(phys, PrefixShard):
        n = padded // cp
        return list(range(j * n, (j + 1) * n))
    if isinstance(phys, RangeSequenceShard):
        c = padded // (2 * cp)
        r = phys.cp_rank
        if padded % (2 * cp) or phys.ranges != ((r * c, (r + 1) * c), ((2 * cp - 1 - r) * c, (2 * cp - r) * c)):
            raise NotImplementedError("P2P CP transport supports contiguous and zigzag shards")
        return list(range(j * c, (j + 1) * c)) + list(range((2 * cp - 1 - j) * c, (2 * cp - j) * c))
    raise NotImplementedError(f"unsupported shard {type(phys).__name__}")


class CPP2PComm:
    def __init__(self, group, device: torch.device, capacity_bytes: int = 32 << 20, timeout_s: float | None = None):
        from .symmetric import SymmetricHeap

        self.group = group
        self.heap = SymmetricHeap(group, device, timeout_s=timeout_s)
        self.n, self.rank = self.heap.size, self.heap.rank
        self.device = device
        self.capacity = capacity_bytes
        self.bufs = [self.heap.alloc(capacity_bytes), self.heap.alloc(capacity_bytes)]
        self.uses = 0
        self._plans: dict = {}

    def next_buffer(self, nbytes: int):
        if nbytes > self.capacity:          # identical shapes on every CP rank -> all grow together
            torch.cuda.synchronize()
            self.heap.barrier()
            self.capacity = max(nbytes, 2 * self.capacity)
            self.bufs = [self.heap.alloc(self.capacity), self.heap.alloc(self.capacity)]
        buf = self.bufs[self.uses % 2]
        self.uses += 1
        return buf

    def plan(self, shards: tuple) -> dict:
        """Index maps for a (prefix blocks..., current) shard tuple (cached)."""
        key = tuple((type(physical_sequence_shard(s)).__name__, s.global_length, s.padded_length) for s in shards)
        p = self._plans.get(key)
        if p is not None:
            return p
        n, me = self.n, self.rank
        local_len = [len(rank_rows(s, me)) for s in shards]
        stg_off = [sum(local_len[:b]) for b in range(len(shards))]
        stg_rows = sum(local_len)
        g_rank, g_row, bank_off = [], [], []
        pos = 0
        for b, s in enumerate(shards):
            last = b == len(shards) - 1
            length = s.padded_length if last else s.global_length
            owner = {}
            for j in range(n):
                for li, g in enumerate(rank_rows(s, j)):
                    owner[g] = (j, stg_off[b] + li)
            bank_off.append(pos)
            for g in range(length):
                j, row = owner[g]
                g_rank.append(j)
                g_row.append(row)
            pos += length
        bank_rows = pos
        # backward: my staging row -> its bank row (padding rows of prefix blocks -> zero row at bank_rows)
        r_row = []
        for b, s in enumerate(shards):
            last = b == len(shards) - 1
            limit = s.padded_length if last else s.global_length
            for g in rank_rows(s, me):
                r_row.append(bank_off[b] + g if g < limit else bank_rows)
        dev = self.device
        p = {
            "stg_rows": stg_rows, "stg_off": stg_off, "local_len": local_len, "bank_rows": bank_rows,
            "bank_off": bank_off,
            "g_rank": torch.tensor(g_rank, dtype=torch.int32, device=dev),
            "g_row_k": torch.tensor(g_row, dtype=torch.int32, device=dev),
            "g_row_v": torch.tensor([r + stg_rows for r in g_row], dtype=torch.int32, device=dev),
            "r_row_k": torch.tensor(r_row, dtype=torch.int32, device=dev),
            "r_row_v": torch.tensor([r + bank_rows + 1 for r in r_row], dtype=torch.int32, device=dev),
        }
        self._plans[key] = p
        return p

    def close(self) -> None:
        self.heap.close()


def cp_comm(group, x: Tensor) -> CPP2PComm | None:
    if _MODE == "nccl" or group is None or not x.is_cuda or x.dtype != torch.bfloat16:
        return None
    n = dist.get_world_size(group)
    local = int(os.environ.get("LOCAL_WORLD_SIZE", dist.get_world_size()))
    if not (1 < n <= 8 and local >= dist.get_world_size()):
        if _MODE == "nvlink":
            raise ValueError("cp_comm='nvlink' needs a single-node CP group of 2..8 GPUs")
        return None
    key = id(group)
    if key not in _COMMS:
        _COMMS[key] = CPP2PComm(group, x.device)
    return _COMMS[key]


def shared_cp_comm(group, device: torch.device) -> CPP2PComm:
    """The group's P2P staging comm (created on first use; shared by every CP transport of the group)."""
    key = id(group)
    if key not in _COMMS:
        _COMMS[key] = CPP2PComm(group, device)
    return _COMMS[key]


def close_all() -> None:
    for c in _COMMS.values():
        c.close()
    _COMMS.clear()


class _P2PKVGather(torch.autograd.Function):
    """``(k_0, v_0, ..., k_cur, v_cur)`` rank-local blocks -> global-order ``bank_k, bank_v``."""

    @staticmethod
    def forward(ctx, comm, plan, *kv):
        m = kernels()
        ks, vs = kv[0::2], kv[1::2]
        width = ks[-1].shape[1] * ks[-1].shape[2]
        rows = plan["stg_rows"]
        buf = comm.next_buffer(2 * rows * width * 2)
        stg = buf.view(torch.bfloat16, 2 * rows * width).view(2 * rows, width)
        torch.cat([k.reshape(-1, width) for k in ks], out=stg[:rows])
        torch.cat([v.reshape(-1, width) for v in vs], out=stg[rows:])
        comm.heap.barrier()
        br = plan["bank_rows"]
        bank_k = torch.empty((br, width), dtype=torch.bfloat16, device=stg.device)
        bank_v = torch.empty((br, width), dtype=torch.bfloat16, device=stg.device)
        m.p2p_gather_rows(bank_k, buf.ptrs, plan["g_rank"], plan["g_row_k"])
        m.p2p_gather_rows(bank_v, buf.ptrs, plan["g_rank"], plan["g_row_v"])
        ctx.comm, ctx.plan, ctx.shapes = comm, plan, [k.shape for k in ks]
        hk, d = ks[-1].shape[1], ks[-1].shape[2]
        return bank_k.view(br, hk, d), bank_v.view(br, hk, d)

    @staticmethod
    def backward(ctx, dbk, dbv):
        m = kernels()
        comm, plan = ctx.comm, ctx.plan
        br, rows = plan["bank_rows"], plan["stg_rows"]
        width = dbk.shape[1] * dbk.shape[2]
        buf = comm.next_buffer(2 * (br + 1) * width * 2)
        stg = buf.view(torch.bfloat16, 2 * (br + 1) * width).view(2 * (br + 1), width)
        stg[:br].copy_(dbk.reshape(br, width))
        stg[br].zero_()
        stg[br + 1:2 * br + 1].copy_(dbv.reshape(br, width))
        stg[2 * br + 1].zero_()
        comm.heap.barrier()
        dk = torch.empty((rows, width), dtype=torch.bfloat16, device=stg.device)
        dv = torch.empty((rows, width), dtype=torch.bfloat16, device=stg.device)
        m.p2p_reduce_rows(dk, buf.ptrs, plan["r_row_k"], False, None)
        m.p2p_reduce_rows(dv, buf.ptrs, plan["r_row_v"], False, None)
        grads = []
        for b, shp in enumerate(ctx.shapes):
            o, n = plan["stg_off"][b], plan["local_len"][b]
            grads += [dk[o:o + n].view(shp), dv[o:o + n].view(shp)]
        return (None, None, *grads)


def p2p_cp_attention(query: Tensor, key: Tensor, value: Tensor, *, prefix_blocks, current_shard, comm: CPP2PComm,
                     softmax_scale: float) -> Tensor:
    """Local-query attention over all prefix blocks and the whole current segment (any CP shard layout
    supported by :func:`rank_rows`)."""
    from ..ops.attention import tree_attention
    from ..tpr.context import SegmentBatchLayout

    shards = tuple(b.shard for b in prefix_blocks) + (current_shard,)
    plan = comm.plan(shards)
    kv = []
    for b in prefix_blocks:
        kv += [b.key, b.value]
    kv += [key, value]
    bank_k, bank_v = _P2PKVGather.apply(comm, plan, *kv)
    P = plan["bank_off"][-1]
    # contiguous runs of local rows -> one tree-attention sequence each (causal self + bank prefix)
    rows = rank_rows(current_shard, comm.rank)
    lens, spans = [], []
    s = 0
    while s < len(rows):
        e = s
        while e + 1 < len(rows) and rows[e + 1] == rows[e] + 1:
            e += 1
        lens.append(e - s + 1)
        spans.append((0, P + rows[s]))
        s = e + 1
    lay_key = ("cp_p2p_layout", tuple(lens), tuple(spans))
    lay = comm._plans.get(lay_key)
    if lay is None:
        lay = SegmentBatchLayout.build(tuple(lens), tuple(spans), device=query.device)
        comm._plans[lay_key] = lay
    o = tree_attention(query, key, value, bank_k, bank_v, lay, softmax_scale=softmax_scale)
    if current_shard.padded_length > current_shard.global_length:
        valid = torch.tensor([g < current_shard.global_length for g in rows], device=o.device)
        o = o * valid[:, None, None].to(o.dtype)
    return o
