"""Ring context parallelism over zigzag shards, with external prefix KV.

Layout: a segment of padded length ``2*cp*c`` is split in ``2*cp`` chunks and
rank r owns chunks ``r`` and ``2cp-1-r``.  Forward: for every KV source
(the ancestors' blocks, root first, then the current segment) the local K/V
block travels once around the ring (``cp-1`` hops, two live buffers); each
visit attends the local queries to the visiting block -- FULL for prefix
blocks and for earlier chunks, CAUSAL on the diagonal, SKIP otherwise -- and
merges the partial ``(o, lse)`` into an FP32 running accumulator (one final
cast).  Backward replays the ring in the same direction with a packet
``(K, V, dK, dV)``: each visited rank adds its queries' dK/dV contribution to
the packet, and after ``cp`` hops the packet is home with the full gradient
of the owner's block.  Constant buffers: 2 (forward), 4 (backward).

On CUDA with a single-node CP group the backend uses the NVLink peer-memory
transport of :mod:`bridge_b200.parallel.cp_p2p` (P2P row gathers into a
global-order bank + the tcgen05 tree-attention kernel + P2P owner reduction of
dK/dV); the NCCL ring below is the baseline and the CPU/gloo path.

Parity: verl/models/mcore/tpr/parallel/ring_attention.py:57-1140
(RingBlockKind, classify_ring_block, zigzag shard, streaming ring forward,
owner reduction of dK/dV in backward, ordinary whole-sequence ring).
"""

from __future__ import annotations

import math
from enum import Enum

import torch
import torch.distributed as dist
from torch import Tensor

from ..tpr.shard import SequenceShard, make_ring_sequence_shard, physical_sequence_shard
from .execution_context import CPAttentionBackendBase, LocalKVBlock, prefix_blocks


class RingBlockKind(str, Enum):
    FULL = "full"
    CAUSAL = "causal"
    SKIP = "skip"


def classify_ring_block(q_range: tuple[int, int], kv_range: tuple[int, int], *, prefix: bool) -> RingBlockKind:
    """Kind of the (query chunk, kv chunk) pair in one segment's global coordinates."""
    if prefix:
        return RingBlockKind.FULL
    (qs, qe), (ks, ke) = q_range, kv_range
    if (qs, qe) == (ks, ke):
        return RingBlockKind.CAUSAL
    if ke <= qs:
        return RingBlockKind.FULL
    if ks >= qe:
        return RingBlockKind.SKIP
    raise ValueError(f"ring chunks must be equal or disjoint, got q={q_range} kv={kv_range}")


# --------------------------------------------------------------------------- block math (FP32)
def block_attention_forward(q: Tensor, k: Tensor, v: Tensor, q_pos: Tensor, k_pos: Tensor, q_valid: Tensor,
                            k_valid: Tensor, scale: float) -> tuple[Tensor, Tensor]:
    """Partial attention of q over one K/V block: ``o [T,Hq,D]`` FP32 (normalised) and ``lse [Hq,T]``."""
    hq, hkv = q.shape[1], k.shape[1]
    qf = q.float().transpose(0, 1)
    kf = k.float().transpose(0, 1).repeat_interleave(hq // hkv, 0)
    vf = v.float().transpose(0, 1).repeat_interleave(hq // hkv, 0)
    s = torch.matmul(qf, kf.transpose(1, 2)) * scale
    allow = (k_pos[None, :] <= q_pos[:, None]) & k_valid[None, :] & q_valid[:, None]
    s = s.masked_fill(~allow[None], float("-inf"))
    lse = torch.logsumexp(s, -1)
    safe = torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))
    p = torch.exp(s - safe[..., None]) * allow[None]
    return torch.matmul(p, vf).transpose(0, 1), lse


def block_attention_backward(q, k, v, do, lse, delta, q_pos, k_pos, q_valid, k_valid, scale):
    """Gradients of one block given the FINAL lse / delta = rowsum(dO*O); returns FP32 dq, dk, dv."""
    hq, hkv = q.shape[1], k.shape[1]
    rep = hq // hkv
    qf = q.float().transpose(0, 1)
    kf = k.float().transpose(0, 1).repeat_interleave(rep, 0)
    vf = v.float().transpose(0, 1).repeat_interleave(rep, 0)
    dof = do.float().transpose(0, 1)
    allow = (k_pos[None, :] <= q_pos[:, None]) & k_valid[None, :] & q_valid[:, None]
    s = torch.matmul(qf, kf.transpose(1, 2)) * scale
    safe = torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))
    p = torch.exp(s - safe[..., None]) * allow[None]
    dp = torch.matmul(dof, vf.transpose(1, 2))
    ds = p * (dp - delta.transpose(0, 1)[..., None])
    dq = torch.matmul(ds, kf).transpose(0, 1) * scale
    dk = torch.matmul(ds.transpose(1, 2), qf) * scale
    dv = torch.matmul(p.transpose(1, 2), dof)
    dk = dk.view(hkv, rep, *dk.shape[1:]).sum(1).transpose(0, 1)
    dv = dv.view(hkv, rep, *dv.shape[1:]).sum(1).transpose(0, 1)
    return dq, dk, dv


def merge_attention(o_a: Tensor | None, lse_a: Tensor | None, o_b: Tensor, lse_b: Tensor):
    """Two-way log-sum-exp merge of normalised partial outputs (FP32)."""
    if o_a is None:
        return o_b, lse_b
    lse = torch.logaddexp(lse_a, lse_b)
    safe = torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))
    wa = torch.exp(lse_a - safe).transpose(0, 1)[..., None]
    wb = torch.exp(lse_b - safe).transpose(0, 1)[..., None]
    return o_a * wa + o_b * wb, lse


# --------------------------------------------------------------------------- transport
def _peer(group, offset: int) -> int:
    n, r = dist.get_world_size(group), dist.get_rank(group)
    return dist.get_global_rank(group, (r + offset) % n)


def ring_exchange(tensors: list[Tensor], group) -> list[Tensor]:
    """Send ``tensors`` to rank+1 and receive the same shapes from rank-1 (one hop)."""
    nxt, prv = _peer(group, 1), _peer(group, -1)
    recv = [torch.empty(t.shape, dtype=t.dtype, device=t.device) for t in tensors]
    ops = []
    for t in tensors:
        ops.append(dist.P2POp(dist.isend, t.contiguous(), nxt, group))
    for t in recv:
        ops.append(dist.P2POp(dist.irecv, t, prv, group))
    for w in dist.batch_isend_irecv(ops):
        w.wait()
    return recv


def zigzag_indices(padded_length: int, rank: int, size: int, device=None) -> Tensor:
    """Global row indices owned by ``rank``: chunks ``rank`` and ``2*size-1-rank`` of ``2*size``."""
    c = padded_length // (2 * size)
    lo, hi = rank * c, (2 * size - 1 - rank) * c
    return torch.cat((torch.arange(lo, lo + c, device=device), torch.arange(hi, hi + c, device=device)))


def _source_positions(shard: SequenceShard, src: int, offset: int, device):
    """Absolute positions and validity of source rank ``src``'s rows of a zigzag-sharded segment."""
    g = zigzag_indices(shard.padded_length, src, shard.cp_size, device)
    return g + offset, g < shard.global_length


def _block_visible(cur_shard: SequenceShard, rank: int, p_cur: int, shard: SequenceShard, src: int,
                   off: int) -> bool:
    """Whether any local query sees any valid key of source ``src`` (the ring's SKIP test), decided from
    the shard geometry on the host -- no device synchronisation per ring step."""
    q_pos, _ = _source_positions(cur_shard, rank, p_cur, None)
    k_pos, k_valid = _source_positions(shard, src, off, None)
    if not bool(k_valid.any()):
        return False
    return int(k_pos[k_valid].min()) <= int(q_pos.max())


class _RingTPRAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, meta, *prefix_flat):
        group, scale, cur_shard, pshards, poffs = meta
        dev = q.device
        rank, n = dist.get_rank(group), dist.get_world_size(group)
        P = sum(s.global_length for s in pshards)
        q_pos, q_valid = _source_positions(cur_shard, rank, P, dev)
        blocks = [(prefix_flat[2 * i], prefix_flat[2 * i + 1], pshards[i], poffs[i]) for i in range(len(pshards))]
        blocks.append((k, v, cur_shard, P))
        o_acc = lse_acc = None
        for bk, bv, shard, off in blocks:
            buf = [bk, bv]
            for step in range(n):
                src = (rank - step) % n
                k_pos, k_valid = _source_positions(shard, src, off, dev)
                if _block_visible(cur_shard, rank, P, shard, src, off):
                    o_b, lse_b = block_attention_forward(q, buf[0], buf[1], q_pos, k_pos, q_valid, k_valid, scale)
                    o_acc, lse_acc = merge_attention(o_acc, lse_acc, o_b, lse_b)
                if step < n - 1:
                    buf = ring_exchange(buf, group)
        o = (o_acc * q_valid[:, None, None]).to(q.dtype)
        ctx.save_for_backward(q, k, v, o, lse_acc, *prefix_flat)
        ctx.meta = meta
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, *prefix_flat = ctx.saved_tensors
        group, scale, cur_shard, pshards, poffs = ctx.meta
        dev = q.device
        rank, n = dist.get_rank(group), dist.get_world_size(group)
        P = sum(s.global_length for s in pshards)
        q_pos, q_valid = _source_positions(cur_shard, rank, P, dev)
        do = do * q_valid[:, None, None].to(do.dtype)
        delta = (do.float() * o.float()).sum(-1)                     # [T, Hq]
        dq = torch.zeros(q.shape, dtype=torch.float32, device=dev)
        blocks = [(prefix_flat[2 * i], prefix_flat[2 * i + 1], pshards[i], poffs[i]) for i in range(len(pshards))]
        blocks.append((k, v, cur_shard, P))
        grads = []
        for bk, bv, shard, off in blocks:
            pkt = [bk, bv, torch.zeros(bk.shape, dtype=torch.float32, device=dev),
                   torch.zeros(bv.shape, dtype=torch.float32, device=dev)]
            for step in range(n):
                src = (rank - step) % n
                k_pos, k_valid = _source_positions(shard, src, off, dev)
                if _block_visible(cur_shard, rank, P, shard, src, off):
                    gq, gk, gv = block_attention_backward(q, pkt[0], pkt[1], do, lse, delta, q_pos, k_pos, q_valid,
                                                          k_valid, scale)
                    dq += gq
                    pkt[2] = pkt[2] + gk
                    pkt[3] = pkt[3] + gv
                pkt = ring_exchange(pkt, group)  # cp hops in total: the packet ends at its owner
            grads.append((pkt[2].to(bk.dtype), pkt[3].to(bv.dtype)))
        dk, dv = grads[-1]
        flat = []
        for gk, gv in grads[:-1]:
            flat += [gk, gv]
        return (dq.to(q.dtype), dk, dv, None, *flat)


def ring_cp_attention(query: Tensor, key: Tensor, value: Tensor, *, prefix_blocks: tuple[LocalKVBlock, ...],
                      current_shard: SequenceShard, cp_group, softmax_scale: float | None) -> Tensor:
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(query.shape[-1])
    pshards = tuple(b.shard for b in prefix_blocks)
    offs, o = [], 0
    for s in pshards:
        offs.append(o)
        o += s.global_length
    flat = []
    for b in prefix_blocks:
        flat += [b.key, b.value]
    return _RingTPRAttention.apply(query, key, value, (cp_group, scale, current_shard, pshards, tuple(offs)), *flat)


def ordinary_ring_cp_attention(query: Tensor, key: Tensor, value: Tensor, *, cp_group, global_length: int,
                               softmax_scale: float | None = None) -> Tensor:
    """Whole-sequence causal ring attention (no external prefix) over zigzag shards: the NVLink P2P
    path (row gathers + tcgen05 tree attention + owner reduction of dK/dV) on a single-node CUDA group,
    the NCCL / gloo ring otherwise."""
    from .cp_p2p import cp_comm, p2p_cp_attention

    shard = make_ring_sequence_shard(global_length, cp_rank=dist.get_rank(cp_group),
                                     cp_size=dist.get_world_size(cp_group))
    comm = cp_comm(cp_group, query)
    if comm is not None:
        scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(query.shape[-1])
        return p2p_cp_attention(query, key, value, prefix_blocks=(), current_shard=shard, comm=comm,
                                softmax_scale=scale)
    return ring_cp_attention(query, key, value, prefix_blocks=(), current_shard=shard, cp_group=cp_group,
                             softmax_scale=softmax_scale)


class RingCPAttentionBackend(CPAttentionBackendBase):
    def attention(self, layer_number: int, query: Tensor, key: Tensor, value: Tensor, *,
                  softmax_scale: float | None = None) -> Tensor:
        from .cp_p2p import cp_comm, p2p_cp_attention

        comm = cp_comm(self.cp_group, query)
        if comm is not None:
            scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(query.shape[-1])
            return p2p_cp_attention(query, key, value, prefix_blocks=self.blocks(layer_number),
                                    current_shard=self.current_shard, comm=comm, softmax_scale=scale)
        return ring_cp_attention(query, key, value, prefix_blocks=self.blocks(layer_number),
                                 current_shard=self.current_shard, cp_group=self.cp_group,
                                 softmax_scale=softmax_scale)


def make_ring_cp_backend(kv_stack, *, expected_layer_numbers, current_shard, cp_group, past_anchors=None):
    blocks = prefix_blocks(kv_stack, expected_layer_numbers, past_anchors)
    prefix = sum(e.state.shard.global_length for e in kv_stack.entries())
    return RingCPAttentionBackend(blocks_by_layer=blocks, current_shard=current_shard, cp_group=cp_group,
                                  global_prefix_length=prefix)
