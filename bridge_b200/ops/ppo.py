"""Vanilla PPO clip / dual-clip policy loss with token-mean aggregation.

Per supervised token with new log-prob ``x``, old log-prob ``o``, advantage
``A`` and optional importance weight ``w``::

    r       = exp(clamp(x - o, -20, 20))
    l1, l2  = -A*r, -A*clamp(r, 1-eps_lo, 1+eps_hi)
    primary = max(l1, l2)
    loss_t  = min(primary, -A*c) if A < 0 else primary        (dual clip, c = 3)
    loss    = sum_t w_t * loss_t / denom                      (global token count)

The CUDA kernel (``csrc/elementwise.cu``) computes the loss sum, dloss/dx and
the clip-fraction / approx-KL / ratio statistics in one pass over the tokens
(one block reduction, no host sync).

Parity: verl ``ppo_loss`` (vanilla, token-mean) as restated in
tests/models/mcore/tpr/parallel/analyze_real_actor_ppo_adjoint.py:36-56.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from ._ext import kernels, on_gpu


@dataclass(frozen=True)
class PPOLossConfig:
    clip_ratio_low: float = 0.2
    clip_ratio_high: float = 0.2
    clip_ratio_c: float = 3.0
    loss_agg_mode: str = "token-mean"
    loss_mode: str = "vanilla"

    def __post_init__(self) -> None:
        if self.loss_mode != "vanilla" or self.loss_agg_mode != "token-mean":
            raise NotImplementedError("TPR PPO supports vanilla policy loss with token-mean aggregation")


def ppo_token_losses_reference(x: Tensor, old: Tensor, adv: Tensor, cfg: PPOLossConfig):
    xf, of, af = x.float(), old.float(), adv.float()
    neg_kl = xf - of
    ratio = torch.exp(torch.clamp(neg_kl, -20.0, 20.0))
    l1 = -af * ratio
    l2 = -af * torch.clamp(ratio, 1.0 - cfg.clip_ratio_low, 1.0 + cfg.clip_ratio_high)
    primary = torch.maximum(l1, l2)
    dual = -af * cfg.clip_ratio_c
    loss = torch.where(af < 0, torch.minimum(primary, dual), primary)
    clipped = (l2 > l1).float()
    dual_clipped = ((af < 0) & (primary > dual)).float()
    return loss, ratio, neg_kl, clipped, dual_clipped


def ppo_loss_reference(x: Tensor, old: Tensor, adv: Tensor, denom: float, cfg: PPOLossConfig,
                       weights: Tensor | None = None):
    loss_t, ratio, neg_kl, clipped, dual = ppo_token_losses_reference(x, old, adv, cfg)
    if weights is not None:
        loss_t = loss_t * weights.float()
    loss = loss_t.sum() / float(denom)
    n = max(int(x.numel()), 1)
    stats = torch.stack([clipped.sum(), dual.sum(), (-neg_kl).sum(), ratio.detach().sum()]) / n
    return loss, stats.detach()


class _PPOLossFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, old, adv, weights, denom, lo, hi, c):
        out, grad, stats = kernels().ppo_loss_fwd(x.float().contiguous(), old.float().contiguous(),
                                                 adv.float().contiguous(),
                                                 weights.float().contiguous() if weights is not None else None,
                                                 float(denom), float(lo), float(hi), float(c))
        ctx.save_for_backward(grad)
        ctx.xdtype = x.dtype
        return out, stats

    @staticmethod
    def backward(ctx, dout, dstats):
        (grad,) = ctx.saved_tensors
        return (grad * dout).to(ctx.xdtype), None, None, None, None, None, None, None


def ppo_loss(x: Tensor, old: Tensor, adv: Tensor, *, denom: float, cfg: PPOLossConfig = PPOLossConfig(),
             weights: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """Return ``(loss, stats)``; ``stats = [clipfrac, dual_clipfrac, approx_kl, mean_ratio]`` (token means)."""
    if x.numel() == 0:
        z = x.sum() * 0.0
        return z, torch.zeros(4, device=x.device)
    if on_gpu(x):
        return _PPOLossFn.apply(x, old, adv, weights, denom, cfg.clip_ratio_low, cfg.clip_ratio_high,
                                cfg.clip_ratio_c)
    return ppo_loss_reference(x, old, adv, denom, cfg, weights)
