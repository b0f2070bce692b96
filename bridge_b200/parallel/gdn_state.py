"""Gated DeltaNet under context parallelism.

Two schedules are provided:

* **head-parallel** (:func:`forward_gdn_cp_with_state`) -- the projected
  ``[q | k | v | z | b | a]`` sections of the contiguous local shard go through
  a sequence->head all-to-all so every rank holds the whole segment for
  ``1/cp`` of the heads (conv channels sliced to match), runs the stateful conv
  and delta rule locally, and returns through head->sequence.  The GDN state is
  head-local: conv ``[B, C/cp, W]``, recurrent ``[B, Hv/cp, K, V]``.
* **sequence-sharded** (:func:`forward_gdn_cp_sequence`, and
  :func:`forward_gdn_cp_tpr` with ``gdn_cp_mode="sequence"``) -- every rank keeps
  its own tokens and all heads.  Each contiguous piece of a rank's rows (one
  for a contiguous shard, two for zigzag) runs the chunked delta rule twice:
  from a zero state (output ``O0``, end state ``C``) and with ``v = 0`` from the
  identity (output ``O_I``, end state ``M``), which gives its affine state map
  ``S_end = M S_start + C`` and ``O = O0 + O_I S_start``.  One all-gather of
  the conv tails (last ``W-1`` inputs, the conv halos) and one of the maps let
  every rank compose the pieces in global order: its pieces' true start
  states, and the segment's final conv / recurrent state, identical on every
  rank.  The backward of each all-gather sums the gradients over ranks, so
  ``dh0`` and the map gradients reach their owners with no extra exchange.
  No token activations cross GPUs (the head-parallel schedule moves the whole
  projection twice per layer); the price is a second delta-rule pass.  On a
  single-node CUDA group the halos and maps (and their gradients) move by NVLink
  P2P (:func:`~bridge_b200.parallel.forest_cp.gather_stack`: one staging write,
  one barrier, peer loads; owner sums in the backward), elsewhere by
  ``all_gather`` / ``all_reduce``.

Parity: verl/models/mcore/tpr/parallel/gdn_state.py:13-104
(gdn_cp_state_shapes, forward_gdn_cp_with_state); the sequence-sharded schedule is new.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist
from torch import Tensor

from ..ops.gdn import causal_conv1d, chunk_gated_delta_rule, gated_rmsnorm, gdn_gates, l2norm
from .ulysses_attention import head_to_sequence, sequence_to_head


_GDN_CP_MODE = os.environ.get("TPR_GDN_CP_MODE", "head")  # head | sequence


def set_gdn_cp_mode(mode: str) -> None:
    """GDN schedule under CP: ``"head"`` (head-parallel exchange, head-local state) or ``"sequence"``
    (sequence-sharded with exchanged state maps, full-head state replicated on every CP rank)."""
    global _GDN_CP_MODE
    if mode not in ("head", "sequence"):
        raise ValueError(f"unknown gdn_cp_mode {mode!r}")
    _GDN_CP_MODE = mode


def gdn_cp_mode() -> str:
    return _GDN_CP_MODE


def gdn_cp_state_shapes(module, cp_size: int, batch: int = 1) -> tuple[tuple[int, ...], tuple[int, ...]]:
    """Head-parallel per-rank state shapes ``(conv, recurrent)``."""
    if module.conv_channels % cp_size or module.hv % cp_size or module.hk % cp_size:
        raise ValueError("GDN heads/channels must divide evenly over CP")
    return (batch, module.conv_channels // cp_size, module.w), (batch, module.hv // cp_size, module.dk, module.dv)


def _split_channels(x: Tensor, sizes: list[int], n: int, r: int) -> Tensor:
    """Select rank ``r``'s 1/n slice of every section of the channel dim."""
    parts = x.split(sizes, dim=-1)
    return torch.cat([p.chunk(n, dim=-1)[r] for p in parts], dim=-1)


def forward_gdn_cp_with_state(module, hidden_local: Tensor, initial_state, cp_group, *,
                              capture_final_state: bool = True):
    """Head-parallel GDN forward of a contiguous local shard; returns ``(out_local, final_state)``."""
    from ..tpr.prefix_state import GDNLayerState

    n, r = dist.get_world_size(cp_group), dist.get_rank(cp_group)
    gdn_cp_state_shapes(module, n)
    kd, vd = module.hk * module.dk, module.hv * module.dv
    proj = module.in_proj(hidden_local)                               # [L_local, 2kd+2vd+2hv]
    sizes = [kd, kd, vd, vd, module.hv, module.hv]
    # Reorder channels so the seq->head exchange hands rank j its slice of every section.
    per_rank = [_split_channels(proj, sizes, n, j) for j in range(n)]
    # [L_local, n, ch/n]: "head" j is rank j's channel slice -> after the exchange [L, 1, ch/n]
    full = sequence_to_head(torch.stack(per_rank, dim=1).contiguous(), cp_group).squeeze(1)
    t = full.shape[0]
    kl, vl, hl = kd // n, vd // n, module.hv // n
    q, k, v, z, b, a = full.split([kl, kl, vl, vl, hl, hl], dim=-1)
    w = _split_channels(module.conv_weight.t(), [kd, kd, vd], n, r).t().contiguous()
    h_conv = initial_state.conv_state if initial_state is not None else None
    h_rec = initial_state.recurrent_state if initial_state is not None else None
    y, conv_final = causal_conv1d(torch.cat([q, k, v], -1), w, None, [0, t], None, h_conv, activation=True)
    q, k, v = y.split([kl, kl, vl], dim=-1)
    hk, hv = module.hk // n, module.hv // n
    q = l2norm(q.reshape(t, hk, module.dk))
    k = l2norm(k.reshape(t, hk, module.dk))
    v = v.reshape(t, hv, module.dv)
    rep = hv // hk
    if rep > 1:
        q, k = q.repeat_interleave(rep, 1), k.repeat_interleave(rep, 1)
    A = module.A_log.chunk(n)[r]
    dt = module.dt_bias.chunk(n)[r]
    g, beta = gdn_gates(a, b, A, dt)
    o, rec_final = chunk_gated_delta_rule(q, k, v, g, beta, [0, t], None, h_rec, scale=module.scale,
                                          chunk_size=module.chunk)
    o = gated_rmsnorm(o, z.reshape(t, hv, module.dv), module.norm_weight, module.eps)
    o_local = head_to_sequence(o.reshape(t, 1, hv * module.dv), cp_group).reshape(hidden_local.shape[0], -1)
    # head_to_sequence restored the sequence shard with channel blocks in rank order == head order
    out = module.out_proj(o_local)
    final = GDNLayerState(conv_final, rec_final) if capture_final_state else None
    return out, final


def affine_chunk_state_map(k: Tensor, v: Tensor, g: Tensor, beta: Tensor, *, chunk_size: int):
    """State map of one sequence shard: ``S_end = M @ S_start + C`` (per head, FP32).

    ``k [L,H,K]``, ``v [L,H,V]``, ``g, beta [L,H]``.  Returns ``M [H,K,K]``, ``C [H,K,V]``.
    """
    L, H, K = k.shape
    V = v.shape[-1]
    M = torch.eye(K, dtype=torch.float32, device=k.device).expand(H, K, K).clone()
    C = torch.zeros((H, K, V), dtype=torch.float32, device=k.device)
    for s in range(0, L, chunk_size):
        e = min(L, s + chunk_size)
        n = e - s
        kc = k[s:e].float().transpose(0, 1)
        vc = v[s:e].float().transpose(0, 1)
        bc = beta[s:e].float().transpose(0, 1)
        G = torch.cumsum(g[s:e].float().transpose(0, 1), -1)
        strict = torch.ones(n, n, dtype=torch.bool, device=k.device).tril(-1)
        diff = G[:, :, None] - G[:, None, :]
        decay = torch.exp(torch.where(strict, diff, torch.full_like(diff, float("-inf"))))
        A = torch.where(strict, decay * torch.matmul(kc, kc.transpose(1, 2)), torch.zeros(1, device=k.device))
        eye = torch.eye(n, device=k.device).expand(H, n, n)
        T = torch.linalg.solve_triangular(eye + bc[:, :, None] * A, eye, upper=False)
        gam = torch.exp(G)
        Wv = torch.matmul(T, bc[:, :, None] * vc)
        Wk = torch.matmul(T, (bc * gam)[:, :, None] * kc)
        kt = (kc * torch.exp(G[:, -1:] - G)[:, :, None]).transpose(1, 2)   # [H, K, n]
        m_chunk = gam[:, -1][:, None, None] * torch.eye(K, device=k.device) - torch.matmul(kt, Wk)
        c_chunk = torch.matmul(kt, Wv)
        M = torch.matmul(m_chunk, M)
        C = torch.matmul(m_chunk, C) + c_chunk
    return M, C


def gdn_sequence_chain_states(M: Tensor, C: Tensor, h0: Tensor, cp_group) -> Tensor:
    """Initial recurrent state of this rank's shard from every rank's affine map (all-gather of maps).

    ``h0`` is the segment's initial state (identical on every rank).  Rank r's
    start state is ``F_{r-1}(...F_0(h0))`` with ``F_i(S) = M_i S + C_i``.
    """
    n, r = dist.get_world_size(cp_group), dist.get_rank(cp_group)
    Ms = [torch.empty_like(M) for _ in range(n)]
    Cs = [torch.empty_like(C) for _ in range(n)]
    dist.all_gather(Ms, M.contiguous(), group=cp_group)
    dist.all_gather(Cs, C.contiguous(), group=cp_group)
    S = h0.float()
    for i in range(r):
        S = torch.matmul(Ms[i], S) + Cs[i]
    return S


_PERM_CACHE: dict = {}


def _shard_permutation(shard, n: int, device):
    """``(pos, valid_len)``: ``pos[g]`` = row of global token ``g`` in the rank-major layout produced by the
    sequence->head exchange (rank j's local rows after rank j-1's), for the valid tokens ``g``."""
    from .cp_p2p import rank_rows

    key = (type(shard).__name__, shard.global_length, shard.padded_length, n, str(device))
    hit = _PERM_CACHE.get(key)
    if hit is not None:
        return hit
    where = {}
    base = 0
    for j in range(n):
        rows = rank_rows(shard, j)
        for li, g in enumerate(rows):
            where[g] = base + li
        base += len(rows)
    valid = shard.global_length
    pos = torch.tensor([where[g] for g in range(valid)], dtype=torch.long, device=device)
    _PERM_CACHE[key] = (pos, valid, base)
    return _PERM_CACHE[key]


def forward_gdn_cp_tpr(module, hidden_local: Tensor, ctx, backend):
    """Head-parallel GDN of one TPR segment whose tokens are CP-sharded (contiguous or zigzag).

    The projected ``[q | k | v | z | b | a]`` channels go through a sequence->head exchange; the rows are
    put back in token order (padding dropped), the stateful conv and chunked delta rule run over the
    whole segment for this rank's 1/cp of the heads from the parent's head-local state, and the output
    returns through head->sequence in the shard's row order.  The final conv / recurrent states are
    head-local, the form every segment of the CP run stores and relays.

    Parity: the six-section cp2hp / hp2cp seam of verl/models/mcore/tpr/parallel/gdn_state.py:25-104
    and gated_delta_net.py:186-202 (un-zigzag inside the exchange).
    """
    from ..tpr.prefix_state import GDNLayerState

    if _GDN_CP_MODE == "sequence":
        return _forward_gdn_cp_tpr_sequence(module, hidden_local, ctx, backend)
    group = backend.cp_group
    n, r = dist.get_world_size(group), dist.get_rank(group)
    gdn_cp_state_shapes(module, n)
    kd, vd = module.hk * module.dk, module.hv * module.dv
    proj = module.in_proj(hidden_local)                               # [L_local, 2kd+2vd+2hv]
    sizes = [kd, kd, vd, vd, module.hv, module.hv]
    per_rank = [_split_channels(proj, sizes, n, j) for j in range(n)]
    full = sequence_to_head(torch.stack(per_rank, dim=1).contiguous(), group).squeeze(1)   # rank-major rows
    pos, t, total = _shard_permutation(backend.current_shard, n, full.device)
    tok = full.index_select(0, pos)                                   # [t, ch/n] in token order
    kl, vl, hl = kd // n, vd // n, module.hv // n
    q, k, v, z, b, a = tok.split([kl, kl, vl, vl, hl, hl], dim=-1)
    w = _split_channels(module.conv_weight.t(), [kd, kd, vd], n, r).t().contiguous()
    init = ctx.get_initial_gdn_state(module.layer_number)
    h_conv = init.conv_state if init is not None else None
    h_rec = init.recurrent_state if init is not None else None
    y, conv_final = causal_conv1d(torch.cat([q, k, v], -1), w, None, [0, t], None, h_conv, activation=True)
    q, k, v = y.split([kl, kl, vl], dim=-1)
    hk, hv = module.hk // n, module.hv // n
    q = l2norm(q.reshape(t, hk, module.dk))
    k = l2norm(k.reshape(t, hk, module.dk))
    v = v.reshape(t, hv, module.dv)
    rep = hv // hk
    if rep > 1:
        q, k = q.repeat_interleave(rep, 1), k.repeat_interleave(rep, 1)
    A = module.A_log.chunk(n)[r]
    dt = module.dt_bias.chunk(n)[r]
    g, beta = gdn_gates(a, b, A, dt)
    o, rec_final = chunk_gated_delta_rule(q, k, v, g, beta, [0, t], None, h_rec, scale=module.scale,
                                          chunk_size=module.chunk)
    o = gated_rmsnorm(o, z.reshape(t, hv, module.dv), module.norm_weight, module.eps).reshape(t, hv * module.dv)
    back = o.new_zeros((total, hv * module.dv)).index_copy(0, pos, o)          # rank-major, padding rows zero
    o_local = head_to_sequence(back.reshape(total, 1, hv * module.dv), group).reshape(hidden_local.shape[0], -1)
    if ctx.capture_gdn_final_state:
        ctx.set_new_gdn_state(module.layer_number, GDNLayerState(conv_final, rec_final))
    return module.out_proj(o_local)


# ------------------------------------------------------------------ sequence-sharded schedule
from .forest_cp import gather_stack  # noqa: E402  (conv halos and state maps: NVLink P2P on CUDA)


class _AllGatherSum(torch.autograd.Function):
    """``[n, *x.shape]`` stack of every rank's ``x``; the backward sums the stacked gradient over ranks
    and returns this rank's slice (every rank may use every slice)."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = dist.get_world_size(group)
        parts = [torch.empty_like(x) for _ in range(n)]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.stack(parts)

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        dist.all_reduce(g, group=ctx.group)
        return g[dist.get_rank(ctx.group)], None


def _valid_pieces(rows: list[int], valid: int) -> list[tuple[int, int, int]]:
    """Maximal runs of consecutive valid global indices in a rank's ``rows``:
    ``(local_start, local_end, global_start)``."""
    out, i = [], 0
    while i < len(rows):
        if rows[i] >= valid:
            i += 1
            continue
        j = i + 1
        while j < len(rows) and rows[j] == rows[j - 1] + 1 and rows[j] < valid:
            j += 1
        out.append((i, j, rows[i]))
        i = j
    return out


def _state_from_tail(tail: Tensor) -> Tensor:
    """Conv state ``[1, C, W]`` (slot 0 unused) from the last ``W-1`` inputs ``[W-1, C]``."""
    return torch.cat([tail.new_zeros(1, tail.shape[1]), tail], 0).t()[None]


def gdn_sequence_sharded(module, proj: Tensor, pieces_by_rank: list[list[tuple[int, int, int]]], group,
                         init=None, capture_final_state: bool = True):
    """Sequence-sharded GDN core.  ``proj [L_local, 2kd+2vd+2hv]`` are this rank's projected rows,
    ``pieces_by_rank[j]`` rank j's valid pieces.  Returns ``(o_local [L_local, hv*dv], final_state)``
    with zero rows where this rank holds padding."""
    from ..tpr.prefix_state import GDNLayerState

    n, r = dist.get_world_size(group), dist.get_rank(group)
    kd, vd, hv, hk, K, V, W = (module.hk * module.dk, module.hv * module.dv, module.hv, module.hk, module.dk,
                               module.dv, module.w)
    cc = 2 * kd + vd
    qkv, z, b, a = proj.split((cc, vd, hv, hv), dim=-1)
    mine = pieces_by_rank[r]
    if any(e - s < W - 1 for pcs in pieces_by_rank for s, e, _ in pcs):
        raise NotImplementedError(f"sequence-sharded GDN needs every shard piece to hold >= {W - 1} tokens")
    P = max(1, max(len(pcs) for pcs in pieces_by_rank))
    order = sorted((g0, j, i) for j, pcs in enumerate(pieces_by_rank) for i, (_, _, g0) in enumerate(pcs))
    # 1. conv halos: every piece's last W-1 pre-conv inputs
    pad_tail = qkv.new_zeros(W - 1, cc)
    tails = torch.stack([qkv[e - (W - 1):e] for s, e, _ in mine] + [pad_tail] * (P - len(mine)))
    all_tails = gather_stack(tails, group)                       # [n, P, W-1, cc]
    h_conv0 = init.conv_state if init is not None else None
    h_rec0 = init.recurrent_state if init is not None else None
    prev = {}
    for k_, (_, j, i) in enumerate(order):
        prev[(j, i)] = order[k_ - 1][1:] if k_ else None
    h0s = []
    for i in range(len(mine)):
        p = prev[(r, i)]
        if p is None:
            h0s.append(h_conv0.reshape(1, cc, W).to(qkv.dtype) if h_conv0 is not None else qkv.new_zeros(1, cc, W))
        else:
            h0s.append(_state_from_tail(all_tails[p[0], p[1]]))
    final_conv = _state_from_tail(all_tails[order[-1][1], order[-1][2]]) if order else None
    if not mine:                       # this rank holds only padding: it still takes part in both gathers
        maps = proj.new_zeros((P, hv, K, K + V), dtype=torch.float32)
        all_maps = gather_stack(maps, group)
        o_local = proj.new_zeros(proj.shape[0], vd)
        S = h_rec0.float() if h_rec0 is not None else proj.new_zeros((1, hv, K, V), dtype=torch.float32)
        for _, j, i in order:
            S = torch.matmul(all_maps[j, i, :, :, :K], S) + all_maps[j, i, :, :, K:]
        return o_local, (GDNLayerState(final_conv, S) if capture_final_state else None)
    cu = [0]
    for s, e, _ in mine:
        cu.append(cu[-1] + e - s)
    t = cu[-1]
    x = torch.cat([qkv[s:e] for s, e, _ in mine])
    y, _ = causal_conv1d(x, module.conv_weight, None, cu, None, torch.cat(h0s), activation=True)
    q, k, v = y.split((kd, kd, vd), dim=-1)
    q = l2norm(q.reshape(t, hk, K))
    k = l2norm(k.reshape(t, hk, K))
    v = v.reshape(t, hv, V)
    if hv // hk > 1:
        q, k = q.repeat_interleave(hv // hk, 1), k.repeat_interleave(hv // hk, 1)
    g, beta = gdn_gates(torch.cat([a[s:e] for s, e, _ in mine]), torch.cat([b[s:e] for s, e, _ in mine]),
                        module.A_log, module.dt_bias)
    # 2. zero-state pass (O0, C) and identity pass with v = 0 (O_I, M), both per piece
    o0, c_end = chunk_gated_delta_rule(q, k, v, g, beta, cu, None, None, scale=module.scale, chunk_size=module.chunk)
    eye = torch.eye(K, dtype=torch.float32, device=q.device).expand(len(mine), hv, K, K).contiguous()
    o_i, m_end = chunk_gated_delta_rule(q, k, torch.zeros_like(k), g, beta, cu, None, eye, scale=module.scale,
                                        chunk_size=module.chunk)
    maps = torch.cat([m_end.float(), c_end.float()], dim=-1)           # [pieces, hv, K, K+V]
    if len(mine) < P:
        maps = torch.cat([maps, maps.new_zeros((P - len(mine),) + maps.shape[1:])])
    all_maps = gather_stack(maps, group)                         # [n, P, hv, K, K+V]
    # 3. compose the pieces in global order
    S = h_rec0.float() if h_rec0 is not None else q.new_zeros((1, hv, K, V), dtype=torch.float32)
    start = {}
    for _, j, i in order:
        start[(j, i)] = S
        S = torch.matmul(all_maps[j, i, :, :, :K], S) + all_maps[j, i, :, :, K:]
    outs = []
    for i in range(len(mine)):
        sl = slice(cu[i], cu[i + 1])
        corr = torch.einsum("thk,hkv->thv", o_i[sl].float(), start[(r, i)][0])
        outs.append((o0[sl].float() + corr).to(o0.dtype))
    o = torch.cat(outs)
    zc = torch.cat([z[s:e] for s, e, _ in mine]).reshape(t, hv, V)
    o = gated_rmsnorm(o, zc, module.norm_weight, module.eps).reshape(t, vd)
    rows = torch.cat([torch.arange(s, e, device=o.device) for s, e, _ in mine])
    o_local = o.new_zeros(proj.shape[0], vd).index_copy(0, rows, o)
    return o_local, (GDNLayerState(final_conv, S) if capture_final_state else None)


def forward_gdn_cp_sequence(module, hidden_local: Tensor, initial_state, cp_group, *,
                            capture_final_state: bool = True):
    """Sequence-sharded GDN forward of a contiguous local shard (equal shards, rank order); returns
    ``(out_local, final_state)`` with the full-head final state on every rank."""
    n = dist.get_world_size(cp_group)
    L = hidden_local.shape[0]
    pieces = [[(0, L, j * L)] for j in range(n)]
    proj = module.in_proj(hidden_local)
    o, final = gdn_sequence_sharded(module, proj, pieces, cp_group, initial_state, capture_final_state)
    return module.out_proj(o), final


def _forward_gdn_cp_tpr_sequence(module, hidden_local: Tensor, ctx, backend):
    from .cp_p2p import rank_rows

    group = backend.cp_group
    n = dist.get_world_size(group)
    shard = backend.current_shard
    pieces = [_valid_pieces(rank_rows(shard, j), shard.global_length) for j in range(n)]
    proj = module.in_proj(hidden_local)
    o, final = gdn_sequence_sharded(module, proj, pieces, group, ctx.get_initial_gdn_state(module.layer_number),
                                    ctx.capture_gdn_final_state)
    if final is not None:
        ctx.set_new_gdn_state(module.layer_number, final)
    return module.out_proj(o)
