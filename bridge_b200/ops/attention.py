"""Tree (prefix-reuse) attention: queries see an external prefix span fully and
their own keys causally.

Layouts are packed token-major: ``q [T, Hq, D]``, ``k, v [T, Hkv, D]`` for the
batch's own tokens and ``pk, pv [P, Hkv, D]`` for the prefix bank.  Segment
``i`` owns rows ``cu[i]:cu[i+1]`` and attends to
``bank[prefix_off[i] : prefix_off[i]+prefix_len[i]]`` plus its own rows
``j <= i`` (right-down aligned causal mask: query ``i`` sees key ``P+j`` for
``j <= i``).  GQA: query head ``h`` reads KV head ``h // (Hq/Hkv)``.

On CUDA the forward and backward are the sm_100a kernels of
``csrc/tree_attention.cu`` (tcgen05/TMEM, FP32 softmax statistics); the prefix
dK/dV of all segments sharing one span are reduced inside the backward
kernel (each CTA owns a KV tile and loops over every query that sees it), so
shared prefix gradients need no atomics and no per-sibling copies.

Parity: verl/models/mcore/tpr/rectangular_attention.py:37-209 (rectangular
right-down causal attention with optional padding mask) -- generalised here to
a packed batch of segments over a shared prefix bank.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import Tensor

from ._ext import kernels, on_gpu

import os

# head_dim 128 runs the tcgen05/TMEM forward; BRIDGE_B200_ATTN=mma selects the mma.sync kernel.
_ATTN_IMPL = os.environ.get("BRIDGE_B200_ATTN", "tcgen05")


# --------------------------------------------------------------------------- reference math
def masked_attention(q: Tensor, k: Tensor, v: Tensor, q_pos: Tensor, k_pos: Tensor, *,
                     k_valid: Tensor | None = None, q_valid: Tensor | None = None,
                     softmax_scale: float, return_lse: bool = False):
    """FP32 attention with the mask ``k_pos <= q_pos`` (and key validity).

    ``q [Sq, Hq, D]``, ``k, v [Sk, Hkv, D]``; returns ``o [Sq, Hq, D]`` in q's
    dtype (and ``lse [Hq, Sq]`` FP32 when asked).  Rows with no visible key
    produce zeros and ``lse = -inf``.
    """
    hq, hkv = q.shape[1], k.shape[1]
    rep = hq // hkv
    qf = q.float().transpose(0, 1)                                   # [Hq, Sq, D]
    kf = k.float().transpose(0, 1).repeat_interleave(rep, dim=0)     # [Hq, Sk, D]
    vf = v.float().transpose(0, 1).repeat_interleave(rep, dim=0)
    s = torch.matmul(qf, kf.transpose(1, 2)) * softmax_scale         # [Hq, Sq, Sk]
    allow = k_pos[None, :] <= q_pos[:, None]
    if k_valid is not None:
        allow = allow & k_valid[None, :]
    if q_valid is not None:
        allow = allow & q_valid[:, None]
    s = s.masked_fill(~allow[None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)                                 # [Hq, Sq]
    p = torch.exp(s - torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))[..., None])
    p = torch.where(allow[None], p, torch.zeros_like(p))
    o = torch.matmul(p, vf).transpose(0, 1).to(q.dtype)
    return (o, lse) if return_lse else o


def rectangular_causal_attention(query: Tensor, key: Tensor, value: Tensor, *, softmax_scale: float | None = None,
                                 dropout_p: float = 0.0, attention_mask: Tensor | None = None) -> Tensor:
    """``Sq <= Skv`` right-down causal attention: query ``i`` sees keys ``<= Skv-Sq+i``.

    ``attention_mask`` (optional, ``[Sq, Skv]`` bool, True = masked) replaces
    the causal rule, as used for padded CP shards.
    """
    if dropout_p != 0.0:
        raise ValueError("TPR attention supports dropout_p=0 only")
    if query.ndim != 3 or key.ndim != 3 or value.ndim != 3:
        raise ValueError("rectangular attention expects [tokens, heads, head_dim] tensors")
    sq, skv = query.shape[0], key.shape[0]
    if sq > skv:
        raise ValueError(f"query length {sq} must not exceed key length {skv}")
    if query.shape[1] % key.shape[1]:
        raise ValueError("query heads must be a multiple of key heads (GQA)")
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(query.shape[-1])
    dev = query.device
    if attention_mask is None:
        q_pos = torch.arange(skv - sq, skv, device=dev)
        k_pos = torch.arange(skv, device=dev)
        if on_gpu(query) and sq > 0:
            lay = _layout_single(sq, skv - sq, dev)
            return tree_attention(query, key[skv - sq:], value[skv - sq:], key[: skv - sq] if skv > sq else None,
                                  value[: skv - sq] if skv > sq else None, lay, softmax_scale=scale)
        return masked_attention(query, key, value, q_pos, k_pos, softmax_scale=scale)
    if attention_mask.shape != (sq, skv) or attention_mask.dtype != torch.bool:
        raise ValueError("attention_mask must be a [Sq, Skv] bool tensor (True = masked)")
    hq, hkv = query.shape[1], key.shape[1]
    qf = query.float().transpose(0, 1)
    kf = key.float().transpose(0, 1).repeat_interleave(hq // hkv, 0)
    vf = value.float().transpose(0, 1).repeat_interleave(hq // hkv, 0)
    s = torch.matmul(qf, kf.transpose(1, 2)) * scale
    s = s.masked_fill(attention_mask[None], float("-inf"))
    p = torch.softmax(s, dim=-1).nan_to_num(0.0)
    return torch.matmul(p, vf).transpose(0, 1).to(query.dtype)


def _layout_single(n: int, prefix: int, device):
    from ..tpr.context import _single_layout

    return _single_layout(n, prefix, device)


def tree_attention_reference(q: Tensor, k: Tensor, v: Tensor, pk: Tensor | None, pv: Tensor | None, layout,
                             *, softmax_scale: float) -> Tensor:
    """Differentiable PyTorch formulation (CPU oracle and GPU library baseline)."""
    outs = []
    cu = 0
    dev = q.device
    for n, (po, pl) in zip(layout.seq_lens, layout.prefix_spans):
        qi, ki, vi = q[cu:cu + n], k[cu:cu + n], v[cu:cu + n]
        if pl:
            ki = torch.cat((pk[po:po + pl], ki))
            vi = torch.cat((pv[po:po + pl], vi))
        if q.is_cuda:
            outs.append(_sdpa_segment(qi, ki, vi, pl, softmax_scale))
        else:
            qp = torch.arange(pl, pl + n, device=dev)
            kp = torch.arange(pl + n, device=dev)
            outs.append(masked_attention(qi, ki, vi, qp, kp, softmax_scale=softmax_scale))
        cu += n
    return outs[0] if len(outs) == 1 else torch.cat(outs)


def _sdpa_segment(q: Tensor, k: Tensor, v: Tensor, prefix: int, scale: float) -> Tensor:
    n, hq, _ = q.shape
    rep = hq // k.shape[1]
    qq = q.transpose(0, 1)[None]
    kk = k.transpose(0, 1).repeat_interleave(rep, 0)[None]
    vv = v.transpose(0, 1).repeat_interleave(rep, 0)[None]
    i = torch.arange(n, device=q.device)[:, None]
    j = torch.arange(prefix + n, device=q.device)[None, :]
    mask = j <= (i + prefix)
    o = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, scale=scale)
    return o[0].transpose(0, 1)


# --------------------------------------------------------------------------- fused path
class _TreeAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, pk, pv, layout, scale):
        m = kernels()
        has_p = pk is not None and layout.prefix_total > 0
        q_, k_, v_ = q.contiguous(), k.contiguous(), v.contiguous()
        pk_ = pk.contiguous() if has_p else q_.new_empty((0, k.shape[1], k.shape[2]))
        pv_ = pv.contiguous() if has_p else q_.new_empty((0, v.shape[1], v.shape[2]))
        fwd = m.tree_attn_fwd_sm100 if (q.shape[-1] == 128 and _ATTN_IMPL == "tcgen05") else m.tree_attn_fwd
        o, lse = fwd(q_, k_, v_, pk_, pv_, layout.cu_seqlens, layout.prefix_offsets, layout.prefix_lengths,
                     layout.max_seqlen, layout.max_prefix, float(scale))
        ctx.save_for_backward(q_, k_, v_, pk_, pv_, o, lse)
        ctx.layout, ctx.scale, ctx.has_p = layout, scale, has_p
        return o

    @staticmethod
    def backward(ctx, do):
        m = kernels()
        q, k, v, pk, pv, o, lse = ctx.saved_tensors
        lay = ctx.layout
        if q.shape[-1] == 128 and _ATTN_IMPL == "tcgen05":
            dq, dk, dv, dpk, dpv = m.tree_attn_bwd_sm100(do.contiguous(), q, k, v, pk, pv, o, lse, lay.cu_seqlens,
                                                         lay.prefix_offsets, lay.prefix_lengths, lay.max_seqlen,
                                                         lay.max_prefix, float(ctx.scale))
            if not ctx.has_p:
                dpk = dpv = None
            return dq, dk, dv, dpk, dpv, None, None
        users, nspans = _prefix_users(lay)
        dq, dk, dv, dpk, dpv = m.tree_attn_bwd(do.contiguous(), q, k, v, pk, pv, o, lse, lay.cu_seqlens,
                                               lay.prefix_offsets, lay.prefix_lengths, lay.max_seqlen,
                                               lay.max_prefix, float(ctx.scale), users, nspans)
        if not ctx.has_p:
            dpk = dpv = None
        return dq, dk, dv, dpk, dpv, None, None


def _prefix_users(layout):
    """CSR map from distinct prefix spans to the segments that read them (cached on the layout)."""
    cached = layout.cache.get("users")
    if cached is not None:
        return cached
    spans: dict[tuple[int, int], list[int]] = {}
    for i, sp in enumerate(layout.prefix_spans):
        if sp[1] > 0:
            spans.setdefault(sp, []).append(i)
    keys = list(spans)
    rowptr, users, span_off, span_len = [0], [], [], []
    for sp in keys:
        users.extend(spans[sp])
        rowptr.append(len(users))
        span_off.append(sp[0])
        span_len.append(sp[1])
    dev = layout.cu_seqlens.device
    t = torch.tensor(rowptr + users + span_off + span_len + [len(keys)], dtype=torch.int32).to(dev, non_blocking=True)
    layout.cache["users"] = (t, len(keys))
    return t, len(keys)


def tree_attention(q: Tensor, k: Tensor, v: Tensor, pk: Tensor | None, pv: Tensor | None, layout,
                   *, softmax_scale: float) -> Tensor:
    if q.ndim != 3 or k.ndim != 3 or v.ndim != 3:
        raise ValueError("tree_attention expects packed [tokens, heads, head_dim] tensors")
    if q.shape[0] != layout.total_tokens or k.shape[0] != q.shape[0]:
        raise ValueError("packed tensors must hold layout.total_tokens rows")
    if q.shape[1] % k.shape[1]:
        raise ValueError("query heads must be a multiple of KV heads")
    if layout.prefix_total and (pk is None or pk.shape[0] < layout.prefix_total):
        raise ValueError("prefix bank is shorter than the layout's spans")
    if on_gpu(q):
        return _TreeAttentionFn.apply(q, k, v, pk, pv, layout, softmax_scale)
    return tree_attention_reference(q, k, v, pk, pv, layout, softmax_scale=softmax_scale)
