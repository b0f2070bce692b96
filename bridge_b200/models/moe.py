"""Mixture-of-experts FFN: softmax top-k router, SwiGLU experts, gated shared expert.

Routing follows the Qwen3-Next form: ``p = softmax(x W_r^T)`` over all experts,
keep the top-k, renormalise them to sum to one; the shared expert output is
scaled by ``sigmoid(x w_g)``.  Under expert parallelism (``ep_group``) every
rank owns ``E / ep`` experts; token rows are exchanged with an all-to-all
(dispatch), run through the local experts as one grouped GEMM over
expert-sorted rows, and exchanged back (combine).

The reference MoE is absent from the TPR extension (it rejects MoE); this is a
new capability of this framework.
"""

from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
from torch import Tensor

from ..ops.activation import swiglu
from ..ops._ext import kernels, on_gpu
from ..ops.gemm import linear
from .config import ModelConfig


class _RouteFn(torch.autograd.Function):
    """Device top-k routing (``csrc/moe_route.cu``): kept weights are a softmax over the k selected
    logits; also returns the stable expert-sorted placement of every routed row."""

    @staticmethod
    def forward(ctx, logits, k):
        idx, w, counts, offsets, pos, order = kernels().moe_route(logits.contiguous(), int(k))
        ctx.save_for_backward(idx, w)
        ctx.E = logits.shape[1]
        ctx.mark_non_differentiable(idx, counts, offsets, pos, order)
        return w, idx, counts, offsets, pos, order

    @staticmethod
    def backward(ctx, dw, *_):
        idx, w = ctx.saved_tensors
        return kernels().moe_route_bwd(idx, w, dw.float().contiguous(), ctx.E), None


class _CombineFn(torch.autograd.Function):
    """``y[t] = sum_j w[t, j] * ys[pos[t, j]]`` (gather-reduce, no atomics) and its backward."""

    @staticmethod
    def forward(ctx, ys, w, pos, t):
        ys = ys.contiguous()
        ctx.save_for_backward(ys, w, pos)
        return kernels().moe_combine(ys, pos, w.contiguous(), int(t))

    @staticmethod
    def backward(ctx, dy):
        ys, w, pos = ctx.saved_tensors
        dys, dw = kernels().moe_combine_bwd(dy.contiguous(), ys, pos, w.contiguous())
        return dys, dw, None, None


def _ep_size(group) -> int:
    return 1 if group is None else dist.get_world_size(group)


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send_counts, recv_counts, group):
        ctx.group, ctx.send, ctx.recv = group, send_counts, recv_counts
        out = x.new_empty((sum(recv_counts), *x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv_counts, send_counts, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = g.new_empty((sum(ctx.send), *g.shape[1:]))
        dist.all_to_all_single(out, g.contiguous(), ctx.send, ctx.recv, group=ctx.group)
        return out, None, None, None


class _GroupedSwiGLUExperts(torch.autograd.Function):
    """All experts' SwiGLU FFNs as two grouped tcgen05 GEMMs over expert-sorted rows (device offsets)."""

    @staticmethod
    def forward(ctx, x, w1, w2, offsets):
        m = kernels()
        h1 = m.grouped_gemm(x, w1, offsets, False)          # [R, 2F] = x W1_e^T
        a = m.swiglu_fwd(h1)                                 # [R, F]
        y = m.grouped_gemm(a, w2, offsets, False)           # [R, H] = a W2_e^T
        ctx.save_for_backward(x, h1, a, w1, w2, offsets)
        return y

    @staticmethod
    def backward(ctx, dy):
        m = kernels()
        x, h1, a, w1, w2, offsets = ctx.saved_tensors
        dy = dy.contiguous()
        da = m.grouped_gemm(dy, w2, offsets, True)          # dy W2_e
        dh1 = m.swiglu_bwd(da, h1)
        dx = m.grouped_gemm(dh1, w1, offsets, True)         # dh1 W1_e
        grads = []
        for w, g_out, g_in in ((w1, dh1, x), (w2, dy, a)):
            main = getattr(w, "main_grad", None)
            if main is not None:                           # accumulate straight into the FP32 main grad
                m.grouped_gemm_wgrad(g_out, g_in, offsets, main)
                grads.append(None)
            else:
                acc = torch.zeros(w.shape, dtype=torch.float32, device=w.device)
                m.grouped_gemm_wgrad(g_out, g_in, offsets, acc)
                grads.append(acc.to(w.dtype))
        return dx, grads[0], grads[1], None


def _grouped_ok(x: Tensor, w1: Tensor, w2: Tensor) -> bool:
    h, f2, f = w1.shape[2], w1.shape[1], w2.shape[2]
    return (on_gpu(x) and x.dtype == torch.bfloat16 and w1.dtype == torch.bfloat16 and h % 64 == 0
            and f2 % 64 == 0 and f % 8 == 0 and w1.shape[0] <= 1024)


def grouped_swiglu_experts(x: Tensor, counts, w1: Tensor, w2: Tensor) -> Tensor:
    """Rows of ``x`` sorted by expert (``counts[e]`` rows each) through expert ``e``'s SwiGLU.

    ``counts`` is a host list or a device tensor; on CUDA the experts run as grouped tcgen05 GEMMs
    whose tile scheduler reads the expert offsets on the device (no host synchronisation).
    """
    if _grouped_ok(x, w1, w2):
        c = counts if isinstance(counts, Tensor) else torch.tensor(counts, device=x.device)
        offsets = torch.zeros(w1.shape[0] + 1, dtype=torch.int32, device=x.device)
        offsets[1:] = torch.cumsum(c.to(x.device), 0).to(torch.int32)
        return _GroupedSwiGLUExperts.apply(x.contiguous(), w1, w2, offsets)
    if isinstance(counts, Tensor):
        counts = counts.tolist()
    outs = []
    s = 0
    for e, n in enumerate(counts):
        if n:
            h = x[s:s + n]
            outs.append(linear(swiglu(linear(h, w1[e])), w2[e]))
        s += n
    if not outs:
        return x.new_zeros((0, w2.shape[1]))
    return torch.cat(outs)


class MoELayer(nn.Module):
    def __init__(self, cfg: ModelConfig, *, ep_group=None, device=None) -> None:
        super().__init__()
        ep = _ep_size(ep_group)
        if cfg.num_experts % ep:
            raise ValueError("num_experts must divide evenly over the EP group")
        self.ep_group = ep_group
        self.num_experts, self.top_k = cfg.num_experts, cfg.moe_top_k
        self.local_experts = cfg.num_experts // ep
        self.ep_rank = 0 if ep_group is None else dist.get_rank(ep_group)
        h, f = cfg.hidden_size, cfg.moe_intermediate_size
        std = cfg.init_std
        self.router = nn.Parameter(torch.randn(cfg.num_experts, h, device=device, dtype=torch.bfloat16) * std)
        self.w1 = nn.Parameter(torch.randn(self.local_experts, 2 * f, h, device=device, dtype=torch.bfloat16) * std)
        self.w2 = nn.Parameter(torch.randn(self.local_experts, h, f, device=device, dtype=torch.bfloat16) * std)
        self.shared = None
        if cfg.shared_expert_intermediate_size:
            fs = cfg.shared_expert_intermediate_size
            self.shared_w1 = nn.Parameter(torch.randn(2 * fs, h, device=device, dtype=torch.bfloat16) * std)
            self.shared_w2 = nn.Parameter(torch.randn(h, fs, device=device, dtype=torch.bfloat16) * std)
            self.shared_gate = nn.Parameter(torch.randn(1, h, device=device, dtype=torch.bfloat16) * std)
            self.shared = True
        self.last_load = None

    def route(self, x: Tensor) -> tuple[Tensor, Tensor]:
        logits = linear(x, self.router).float()
        probs = torch.softmax(logits, dim=-1)
        w, idx = torch.topk(probs, self.top_k, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        return w, idx

    def forward(self, x: Tensor) -> Tensor:
        t, h = x.shape
        device_route = on_gpu(x) and x.dtype == torch.bfloat16 and h % 8 == 0
        if device_route:
            # routing, expert sort and the combine run as this framework's kernels
            logits = linear(x, self.router).float()
            w, idx, counts_all, _, pos, order = _RouteFn.apply(logits, self.top_k)
            rows = order.long() // self.top_k
        else:
            w, idx = self.route(x)
            flat_e = idx.reshape(-1)                                   # [T*k]
            order = torch.argsort(flat_e, stable=True)
            rows = order // self.top_k
            counts_all = torch.bincount(flat_e, minlength=self.num_experts)
        xs = x.index_select(0, rows)
        self.last_load = counts_all.detach()
        ep = _ep_size(self.ep_group)
        comm = None
        if ep > 1:
            from ..parallel.ep_p2p import ep_comm, ep_moe_experts

            comm = ep_comm(self.ep_group, xs)
        if ep == 1:
            y_sorted = grouped_swiglu_experts(xs, counts_all, self.w1, self.w2)
        elif comm is not None:                 # NVLink P2P dispatch / combine around the grouped GEMMs
            y_sorted = ep_moe_experts(xs, counts_all, comm, self.local_experts,
                                      lambda xr, cl: grouped_swiglu_experts(xr, cl, self.w1, self.w2))
        else:
            per_rank = counts_all.view(ep, self.local_experts)
            send = per_rank.sum(1)
            recv_matrix = torch.empty_like(per_rank)
            dist.all_to_all_single(recv_matrix, per_rank.contiguous(), group=self.ep_group)
            send_l, recv_l = send.tolist(), recv_matrix.sum(1).tolist()
            xr = _AllToAll.apply(xs, send_l, recv_l, self.ep_group)
            # Received rows are grouped by source rank then by local expert: re-sort by expert.
            rm = recv_matrix.tolist()
            src_starts, s = [], 0
            for r in range(ep):
                src_starts.append(s)
                s += sum(rm[r])
            perm = []
            counts_local = []
            for e in range(self.local_experts):
                n_e = 0
                for r in range(ep):
                    start = src_starts[r] + sum(rm[r][:e])
                    perm.extend(range(start, start + rm[r][e]))
                    n_e += rm[r][e]
                counts_local.append(n_e)
            perm_t = torch.tensor(perm, device=x.device, dtype=torch.long)
            ye = grouped_swiglu_experts(xr.index_select(0, perm_t), counts_local, self.w1, self.w2)
            inv = torch.empty_like(perm_t)
            inv[perm_t] = torch.arange(perm_t.numel(), device=x.device)
            y_sorted = _AllToAll.apply(ye.index_select(0, inv), recv_l, send_l, self.ep_group)
        if device_route:
            y = _CombineFn.apply(y_sorted, w.reshape(-1), pos, t)
        else:
            gate = w.reshape(-1).index_select(0, order).to(y_sorted.dtype)[:, None]
            y = torch.zeros((t, h), device=x.device, dtype=torch.float32)
            y.index_add_(0, rows, (y_sorted * gate).float())
            y = y.to(x.dtype)
        if self.shared:
            sh = linear(swiglu(linear(x, self.shared_w1)), self.shared_w2)
            y = y + sh * torch.sigmoid(linear(x, self.shared_gate).float()).to(sh.dtype)
        return y
