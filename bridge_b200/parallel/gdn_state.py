"""Gated DeltaNet under context parallelism.

Two schedules are provided:

* **head-parallel** (:func:`forward_gdn_cp_with_state`) -- the projected
  ``[q | k | v | z | b | a]`` sections of the contiguous local shard go through
  a sequence->head all-to-all so every rank holds the whole segment for
  ``1/cp`` of the heads (conv channels sliced to match), runs the stateful conv
  and delta rule locally, and returns through head->sequence.  The GDN state is
  head-local: conv ``[B, C/cp, W]``, recurrent ``[B, Hv/cp, K, V]``.
* **sequence chain** (:func:`gdn_sequence_chain_states`) -- sequence-sharded:
  rank r computes its shard's affine state map ``S_end = M_r S_start + C_r``
  (FP32 ``[H, K, K]`` / ``[H, K, V]``), ranks exchange these maps, and each
  rank composes the prefix of maps to get its true initial state; the conv
  tail (last ``W-1`` inputs) is handed to the next rank the same way.  Backward
  mirrors it for ``dh0``.  This avoids the all-to-all entirely and is the
  schedule used with TP x CP.

Parity: verl/models/mcore/tpr/parallel/gdn_state.py:13-104
(gdn_cp_state_shapes, forward_gdn_cp_with_state); the sequence chain is new.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

from ..ops.gdn import causal_conv1d, chunk_gated_delta_rule, gated_rmsnorm, gdn_gates, l2norm
from .ulysses_attention import head_to_sequence, sequence_to_head


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
