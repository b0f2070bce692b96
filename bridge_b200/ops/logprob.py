"""Fused LM head + temperature-scaled log-prob (+ entropy) over the vocabulary.

For ``U`` selected hidden rows ``h [U, H]`` and a (possibly vocab-parallel)
head ``W [V_local, H]``:  ``z = (h @ W^T) / T``,
``logp[u] = z[u, target[u]] - logsumexp(z[u])`` and
``entropy[u] = logsumexp(z[u]) - sum_v softmax(z[u])_v z[u, v]``.

The CUDA path computes the logits tile by tile of rows (``chunk_rows``), runs
one kernel per chunk that produces the per-row partial statistics
``(max, sum exp, target logit, sum exp*z)`` (combined across TP ranks with one
all-reduce of ``[U, 4]`` partials), and in backward rewrites the saved logits
*in place* into ``dL/dlogits = (dlogp*(onehot - p) - dent*p*(z - E[z])) / T`` before
the two GEMMs -- the ``[U, V]`` FP32 softmax is never materialised.

:func:`fused_lm_head_ppo` goes one step further for the PPO objective: the loss gradient of every
selected row is known as soon as its log-prob is (old log-prob, advantage and the global denominator
are inputs), so the forward itself rewrites each logits chunk into ``dL/dlogits``, runs the two
backward GEMMs (``dh`` saved, ``dW`` accumulated into the FP32 main gradient) and frees the chunk.
Nothing of size ``[U, V]`` outlives the call; backward only scales the saved ``dh``.

Parity: verl vocab_parallel_log_probs_from_logits / vocab_parallel_entropy as
called from verl/models/mcore/tpr/objective_adapter.py:35-44,206-273.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
from torch import Tensor

from ._ext import kernels, on_gpu
from .gemm import gemm


def logprob_entropy_reference(logits: Tensor, targets: Tensor, temperature: Tensor | float = 1.0,
                              *, with_entropy: bool = False, tp_group=None, vocab_start: int = 0):
    """Differentiable reference on (possibly vocab-sharded) logits ``[U, V_local]``."""
    t = temperature if isinstance(temperature, Tensor) else torch.full((logits.shape[0],), float(temperature),
                                                                       device=logits.device)
    z = logits.float() / t.float()[:, None]
    if tp_group is None or dist.get_world_size(tp_group) == 1:
        lse = torch.logsumexp(z, dim=-1)
        lp = z.gather(1, targets[:, None]).squeeze(1) - lse
        ent = None
        if with_entropy:
            p = torch.softmax(z, dim=-1)
            ent = lse - (p * z).sum(-1)
        return lp, ent
    lp, ent = _VocabParallelLogProb.apply(z, targets, vocab_start, tp_group, with_entropy)
    return lp, (ent if with_entropy else None)


class _VocabParallelLogProb(torch.autograd.Function):
    """Vocab-parallel log-prob/entropy on FP32 scaled logits (reference math + TP all-reduces)."""

    @staticmethod
    def forward(ctx, z, targets, vocab_start, group, with_entropy):
        vloc = z.shape[1]
        m = z.max(dim=1).values
        dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
        e = torch.exp(z - m[:, None])
        local = targets - vocab_start
        inside = (local >= 0) & (local < vloc)
        tz = torch.where(inside, z.gather(1, local.clamp(0, vloc - 1)[:, None]).squeeze(1), torch.zeros_like(m))
        stats = torch.stack([e.sum(1), tz, (e * z).sum(1)], dim=1)
        dist.all_reduce(stats, group=group)
        s, tz, ez = stats.unbind(1)
        lse = m + torch.log(s)
        lp = tz - lse
        ent = lse - ez / s if with_entropy else None
        ctx.save_for_backward(z, lse, (ez / s), local, inside)
        ctx.with_entropy = with_entropy
        return (lp, ent) if with_entropy else (lp, lp.new_zeros(0))

    @staticmethod
    def backward(ctx, dlp, dent):
        z, lse, ez, local, inside = ctx.saved_tensors
        p = torch.exp(z - lse[:, None])
        g = -p * dlp[:, None]
        rows = torch.nonzero(inside).flatten()
        g[rows, local[rows]] += dlp[rows]
        if ctx.with_entropy and dent is not None and dent.numel():
            g = g - dent[:, None] * p * (z - ez[:, None])
        return g, None, None, None, None


class _FusedHeadLogProbFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, weight, targets, inv_temp, vocab_start, tp_group, with_entropy, chunk_rows):
        m = kernels()
        u = h.shape[0]
        stats = torch.empty((u, 4), device=h.device, dtype=torch.float32)
        logits_chunks = []
        for s in range(0, u, chunk_rows):
            e = min(u, s + chunk_rows)
            lg = gemm(h[s:e], weight)                                 # [c, V_local] bf16 (tcgen05)
            m.logprob_stats(lg, targets[s:e], inv_temp[s:e], int(vocab_start), stats[s:e])
            logits_chunks.append(lg)
        if tp_group is not None and dist.get_world_size(tp_group) > 1:
            stats = _combine_tp_stats(stats, tp_group)
        lse, lp, ent, ez = m.logprob_finalize(stats)
        ctx.save_for_backward(h, weight, targets, inv_temp, lse, ez)
        ctx.logits = logits_chunks
        ctx.vocab_start, ctx.chunk_rows, ctx.with_entropy = vocab_start, chunk_rows, with_entropy
        return lp, ent

    @staticmethod
    def backward(ctx, dlp, dent):
        m = kernels()
        h, weight, targets, inv_temp, lse, ez = ctx.saved_tensors
        dlp = dlp.float().contiguous() if dlp is not None else torch.zeros_like(lse)
        dent = dent.float().contiguous() if (dent is not None and ctx.with_entropy) else None
        dh = torch.empty_like(h)
        dw = None
        main = getattr(weight, "main_grad", None)
        for i, lg in enumerate(ctx.logits):
            s = i * ctx.chunk_rows
            e = s + lg.shape[0]
            m.logprob_grad_inplace(lg, targets[s:e], inv_temp[s:e], lse[s:e], ez[s:e], dlp[s:e],
                                   dent[s:e] if dent is not None else None, int(ctx.vocab_start))
            dh[s:e] = gemm(lg, weight, b_mn=True)                      # dlogits @ W
            if main is not None:                                       # W.main_grad += dlogits^T h
                gemm(lg, h[s:e].contiguous(), a_mn=True, b_mn=True, out=main, accumulate=True)
            else:
                part = gemm(lg, h[s:e].contiguous(), a_mn=True, b_mn=True)
                dw = part if dw is None else dw.add_(part)
        ctx.logits = None
        return dh, dw, None, None, None, None, None, None


class _FusedHeadPPOFn(torch.autograd.Function):
    """LM head + log-prob + PPO loss with the head's backward done inside the forward.

    ``grad_scale`` is the factor the caller multiplies the loss by before ``backward`` (the
    executor's loss scale).  The weight gradient for that factor is accumulated into ``main_grad``
    during the forward; ``dh`` is saved and scaled by ``dL / grad_scale`` in backward."""

    @staticmethod
    def forward(ctx, h, weight, targets, inv_temp, inverse, old, adv, weights, denom, lo, hi, c, vocab_start,
                tp_group, with_entropy, chunk_rows, grad_scale):
        m = kernels()
        u = h.shape[0]
        stats = torch.empty((u, 4), device=h.device, dtype=torch.float32)
        chunks = []
        for s in range(0, u, chunk_rows):
            e = min(u, s + chunk_rows)
            lg = gemm(h[s:e], weight)                                 # [c, V_local] bf16 (tcgen05)
            m.logprob_stats(lg, targets[s:e], inv_temp[s:e], int(vocab_start), stats[s:e])
            chunks.append(lg)
        if tp_group is not None and dist.get_world_size(tp_group) > 1:
            stats = _combine_tp_stats(stats, tp_group)
        lse, lp_u, ent_u, ez = m.logprob_finalize(stats)
        x = lp_u.index_select(0, inverse)
        loss, g_ref, pstats = m.ppo_loss_fwd(x.contiguous(), old.float().contiguous(), adv.float().contiguous(),
                                             weights.float().contiguous() if weights is not None else None,
                                             float(denom), float(lo), float(hi), float(c))
        dlp = torch.zeros_like(lp_u).index_add_(0, inverse, g_ref)
        dlp.mul_(float(grad_scale))
        dh = torch.empty_like(h)
        main = getattr(weight, "main_grad", None)
        dw = None
        for i, lg in enumerate(chunks):
            s = i * chunk_rows
            e = s + lg.shape[0]
            m.logprob_grad_inplace(lg, targets[s:e], inv_temp[s:e], lse[s:e], ez[s:e], dlp[s:e], None,
                                   int(vocab_start))
            dh[s:e] = gemm(lg, weight, b_mn=True)                      # dlogits @ W
            if main is not None:                                       # W.main_grad += dlogits^T h
                gemm(lg, h[s:e].contiguous(), a_mn=True, b_mn=True, out=main, accumulate=True)
            else:
                part = gemm(lg, h[s:e].contiguous(), a_mn=True, b_mn=True).float()
                dw = part if dw is None else dw.add_(part)
            chunks[i] = None                                           # free the chunk now
        ctx.save_for_backward(dh, dw if dw is not None else dh.new_empty(0))
        ctx.grad_scale, ctx.has_dw = float(grad_scale), dw is not None
        ctx.mark_non_differentiable(pstats, lp_u, ent_u)
        return loss, pstats, lp_u, ent_u

    @staticmethod
    def backward(ctx, dloss, dstats, dlp, dent):
        dh, dw = ctx.saved_tensors
        f = dloss.float() / ctx.grad_scale
        gh = (dh.float() * f).to(dh.dtype)
        gw = (dw * f).to(torch.bfloat16) if ctx.has_dw else None
        return (gh, gw) + (None,) * 15


def fused_lm_head_ppo(h: Tensor, weight: Tensor, targets: Tensor, temperature: Tensor, inverse: Tensor, old: Tensor,
                      adv: Tensor, weights: Tensor | None, *, denom: float, clip_low: float, clip_high: float,
                      clip_c: float, vocab_start: int = 0, tp_group=None, with_entropy: bool = False,
                      chunk_rows: int = 4096, grad_scale: float = 1.0):
    """PPO loss of refs ``lp[inverse]`` where ``lp`` are the log-probs of the unique rows ``h`` (CUDA).

    Returns ``(loss, stats, lp_unique, entropy_unique)``; only ``loss`` is differentiable, and its
    backward must be called with ``grad_scale`` as the loss gradient (see :class:`_FusedHeadPPOFn`)."""
    inv = (1.0 / temperature.float()).contiguous()
    loss, stats, lp, ent = _FusedHeadPPOFn.apply(h.contiguous(), weight, targets.contiguous(), inv,
                                                 inverse.contiguous(), old, adv, weights, denom, clip_low, clip_high,
                                                 clip_c, vocab_start, tp_group, with_entropy, chunk_rows, grad_scale)
    return loss, stats, lp, (ent if with_entropy else None)


def _combine_tp_stats(stats: Tensor, group) -> Tensor:
    """Merge per-rank ``(max, sumexp, target, sum exp*z)`` partials across the TP group."""
    m = stats[:, 0].clone()
    dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
    scale = torch.exp(stats[:, 0] - m)
    merged = torch.stack([stats[:, 1] * scale, stats[:, 2], stats[:, 3] * scale], dim=1)
    dist.all_reduce(merged, group=group)
    return torch.cat([m[:, None], merged], dim=1)


def fused_lm_head_logprob(h: Tensor, weight: Tensor, targets: Tensor, temperature: Tensor, *,
                          vocab_start: int = 0, tp_group=None, with_entropy: bool = False,
                          chunk_rows: int = 4096) -> tuple[Tensor, Tensor | None]:
    """``logp, entropy`` of ``targets`` under ``softmax((h @ W^T) / T)``, never storing FP32 logits."""
    if on_gpu(h):
        inv = (1.0 / temperature.float()).contiguous()
        lp, ent = _FusedHeadLogProbFn.apply(h.contiguous(), weight, targets.contiguous(), inv, vocab_start,
                                            tp_group, with_entropy, chunk_rows)
        return lp, (ent if with_entropy else None)
    logits = torch.matmul(h, weight.t())
    return logprob_entropy_reference(logits, targets, temperature, with_entropy=with_entropy, tp_group=tp_group,
                                     vocab_start=vocab_start)
