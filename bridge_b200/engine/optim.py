"""Mixed-precision AdamW over one flat parameter arena.

Layout (per dtype group, bf16 model parameters):

* ``model params`` -- views into one contiguous bf16 arena (what the kernels read);
* ``master``       -- FP32 copy of the arena;
* ``main_grad``    -- FP32 gradient accumulator; after every backward each
                      parameter's bf16 ``.grad`` is folded into it by a
                      post-accumulate hook and released, so gradients
                      accumulate in FP32 across the forest's chunks;
* ``exp_avg / exp_avg_sq`` -- FP32 Adam moments.

The update is one fused CUDA kernel over the whole arena (decoupled weight
decay, bias correction, FP32 math, writes master + bf16 params in the same
pass).  Non-bf16 parameters (e.g. FP32 GDN ``A_log``) live in a second FP32
arena handled by the same kernel.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor, nn

from ..ops._ext import kernels, on_gpu


@dataclass(frozen=True)
class AdamWConfig:
    lr: float = 1e-6
    betas: tuple[float, float] = (0.9, 0.999)
    eps: float = 1e-8
    weight_decay: float = 0.01
    grad_clip: float = 1.0


class _Arena:
    def __init__(self, params: list[nn.Parameter], dtype, device) -> None:
        self.params = params
        n = sum(p.numel() for p in params)
        self.numel = n
        self.data = torch.empty(n, dtype=dtype, device=device)
        self.master = torch.empty(n, dtype=torch.float32, device=device)
        self.main_grad = torch.zeros(n, dtype=torch.float32, device=device)
        self.m = torch.zeros(n, dtype=torch.float32, device=device)
        self.v = torch.zeros(n, dtype=torch.float32, device=device)
        off = 0
        self.offsets = []
        for p in params:
            k = p.numel()
            self.data[off:off + k].copy_(p.data.reshape(-1))
            p.data = self.data[off:off + k].view_as(p)
            p.main_grad = self.main_grad[off:off + k].view(p.shape)  # type: ignore[attr-defined]
            self.offsets.append(off)
            off += k
        self.master.copy_(self.data.float())


class MixedPrecisionAdamW:
    """FP32-master AdamW for a module whose parameters are bf16 (or fp32)."""

    def __init__(self, module: nn.Module, cfg: AdamWConfig = AdamWConfig()) -> None:
        self.cfg = cfg
        params = [p for p in module.parameters() if p.requires_grad]
        dev = params[0].device
        self.arenas = []
        for dt in (torch.bfloat16, torch.float32):
            group = [p for p in params if p.dtype == dt]
            if group:
                self.arenas.append(_Arena(group, dt, dev))
        other = [p for p in params if p.dtype not in (torch.bfloat16, torch.float32)]
        if other:
            raise TypeError(f"unsupported parameter dtype {other[0].dtype}")
        self.step_count = 0
        self._hooks = [p.register_post_accumulate_grad_hook(self._fold) for a in self.arenas for p in a.params]

    @staticmethod
    def _fold(p: Tensor) -> None:
        if p.grad is not None:
            p.main_grad.add_(p.grad.view(p.main_grad.shape))
            p.grad = None

    def zero_grad(self) -> None:
        for a in self.arenas:
            a.main_grad.zero_()
            for p in a.params:
                p.grad = None

    def grad_buffers(self) -> list[Tensor]:
        return [a.main_grad for a in self.arenas]

    def grad_norm(self) -> Tensor:
        grads = [a.main_grad for a in self.arenas]
        if grads and all(on_gpu(g) and g.dtype == torch.float32 and g.is_contiguous() for g in grads):
            acc = torch.zeros(1, dtype=torch.float32, device=grads[0].device)
            for i, g in enumerate(grads):     # one read of each FP32 arena, no squared copy
                kernels().sumsq_into(g, acc, i > 0)
            return torch.sqrt(acc[0])
        sq = [g.float().pow(2).sum() for g in grads]
        return torch.sqrt(torch.stack(sq).sum())

    def step(self, *, grad_norm: Tensor | None = None) -> Tensor:
        """One AdamW update; returns the pre-clip gradient norm (device scalar, no host sync)."""
        c = self.cfg
        self.step_count += 1
        norm = self.grad_norm() if grad_norm is None else grad_norm
        clip = torch.clamp(c.grad_clip / (norm + 1e-6), max=1.0) if c.grad_clip > 0 else torch.ones_like(norm)
        b1, b2 = c.betas
        bc1 = 1.0 - b1 ** self.step_count
        bc2 = 1.0 - b2 ** self.step_count
        for a in self.arenas:
            if on_gpu(a.master):
                kernels().adamw_step(a.master, a.data, a.main_grad, a.m, a.v, clip, float(c.lr), float(b1), float(b2),
                                     float(c.eps), float(c.weight_decay), float(bc1), float(bc2))
            else:
                g = a.main_grad * clip
                a.m.mul_(b1).add_(g, alpha=1 - b1)
                a.v.mul_(b2).addcmul_(g, g, value=1 - b2)
                denom = (a.v / bc2).sqrt_().add_(c.eps)
                a.master.mul_(1 - c.lr * c.weight_decay).addcdiv_(a.m / bc1, denom, value=-c.lr)
                a.data.copy_(a.master.to(a.data.dtype))
        return norm

    # -- checkpoint support
    def state_dict(self) -> dict:
        return {"step": self.step_count, "arenas": [{"master": a.master, "m": a.m, "v": a.v} for a in self.arenas]}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        for a, s in zip(self.arenas, sd["arenas"]):
            a.master.copy_(s["master"])
            a.m.copy_(s["m"])
            a.v.copy_(s["v"])
            a.data.copy_(a.master.to(a.data.dtype))


_MAX_BUCKETS = 512          # flag slots per peer (bucket ids are global across arenas)
_PARTIALS_PER_BUCKET = 128  # norm partials (= reduce-scatter blocks) per bucket


def bucket_groups(module: nn.Module) -> list[tuple[object, list[nn.Parameter]]]:
    """Parameters cut into gradient buckets in ``module.parameters()`` order: one bucket per decoder
    layer (label = layer index), the embedding (label ``"embed"``) and the rest (``"tail"``).  A module
    without ``layers`` gives one bucket per top-level child."""
    params = [p for p in module.parameters() if p.requires_grad]
    owner: dict[int, object] = {}
    layers = getattr(module, "layers", None)
    if layers is not None:
        for i, layer in enumerate(layers):
            for p in layer.parameters():
                owner[id(p)] = i
        emb = getattr(module, "embed_tokens", None)
        for p in (emb.parameters() if emb is not None else ()):
            owner[id(p)] = "embed"
    else:
        for name, child in module.named_children():
            for p in child.parameters():
                owner.setdefault(id(p), name)
    groups: list[tuple[object, list[nn.Parameter]]] = []
    for p in params:
        label = owner.get(id(p), "tail")
        if groups and groups[-1][0] == label:
            groups[-1][1].append(p)
        else:
            groups.append((label, [p]))
    return groups


class _ShardedArena:
    """Arena whose bf16 (or FP32) parameters and FP32 gradients live in symmetric peer memory, cut into
    buckets (groups of whole parameters, each padded to a multiple of 8 x N elements).  Rank r owns the
    r-th N-th of EVERY bucket, so each bucket's reduce-scatter involves all ranks equally and can run as
    soon as the bucket's gradients are final.  The FP32 master and Adam moments hold only this rank's
    pieces, concatenated in bucket order."""

    def __init__(self, groups: list[tuple[object, list[nn.Parameter]]], dtype, heap) -> None:
        n, r = heap.size, heap.rank
        self.params = [p for _, g in groups for p in g]
        self.numel = sum(p.numel() for p in self.params)
        self.buckets = []          # (label, off, padded, sub, lo)
        off = lo = 0
        for label, g in groups:
            size = sum(p.numel() for p in g)
            padded = max(8 * n, -(-size // (8 * n)) * 8 * n)
            self.buckets.append((label, off, padded, padded // n, lo))
            off += padded
            lo += padded // n
        total, self.shard = off, lo
        esize = torch.tensor([], dtype=dtype).element_size()
        self.data_buf = heap.alloc(total * esize)
        self.grad_buf = heap.alloc(total * 4)
        self.data = self.data_buf.view(dtype, total)
        self.main_grad = self.grad_buf.view(torch.float32, total)
        self.bf16 = dtype == torch.bfloat16
        self.param_ranges = []     # (arena offset, numel) per parameter, in order
        for (label, boff, _, _, _), (_, g) in zip(self.buckets, groups):
            o = boff
            for p in g:
                k = p.numel()
                self.data[o:o + k].copy_(p.data.reshape(-1))
                p.data = self.data[o:o + k].view_as(p)
                p.main_grad = self.main_grad[o:o + k].view(p.shape)  # type: ignore[attr-defined]
                self.param_ranges.append((o, k))
                o += k
        self.master = torch.cat([self.data[b + r * sub:b + (r + 1) * sub] for _, b, _, sub, _ in self.buckets]).float()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)

    def own_range(self, i: int, rank: int) -> tuple[int, int, int]:
        """``(arena offset, count, local offset)`` of ``rank``'s piece of bucket ``i``."""
        _, off, _, sub, lo = self.buckets[i]
        return off + rank * sub, sub, lo

    def to_param_order(self, pieces: list[Tensor]) -> Tensor:
        """Per-rank shard vectors -> the parameters' values concatenated in parameter order."""
        full = torch.empty(self.buckets[-1][1] + self.buckets[-1][2], dtype=pieces[0].dtype, device=pieces[0].device)
        for j, piece in enumerate(pieces):
            for _, off, _, sub, lo in self.buckets:
                full[off + j * sub:off + (j + 1) * sub] = piece[lo:lo + sub]
        return torch.cat([full[o:o + k] for o, k in self.param_ranges])

    def from_param_order(self, flat: Tensor, rank: int) -> Tensor:
        """Inverse of :meth:`to_param_order` for one rank (padding = 0)."""
        full = torch.zeros(self.buckets[-1][1] + self.buckets[-1][2], dtype=torch.float32, device=flat.device)
        s = 0
        for o, k in self.param_ranges:
            full[o:o + k] = flat[s:s + k]
            s += k
        return torch.cat([full[off + rank * sub:off + (rank + 1) * sub] for _, off, _, sub, _ in self.buckets])


class ShardedNVLinkAdamW(MixedPrecisionAdamW):
    """Data-parallel AdamW whose gradient reduction and parameter broadcast are NVLink P2P kernels.

    Per bucket: the compute stream marks the bucket final on every peer (``dp_bucket_signal``); a
    reduce-scatter stream waits until every peer marked it (``dp_bucket_wait``, bounded) and pulls this
    rank's piece from every peer (FP32, fixed rank order, scale 1/N) with the norm partials.  When the
    executor arms the overlap before its last backward (:meth:`arm_overlap`), buckets are issued from
    per-layer gradient hooks while earlier layers still compute; ``step()`` issues whatever is left,
    joins the stream, and then runs: payload barrier carrying the norm partials -> AdamW on this
    rank's pieces with the new parameters stored into every peer's arena -> barrier.  Master weights and
    Adam moments are sharded (1/N of the FP32 optimizer state per rank).  Replicated-but-partial
    gradients of TP-sharded layers (``tp_partial_grad``) are summed over ``tp_group`` when their bucket is
    issued, before the data-parallel reduction reads them.
    """

    handles_tp_partial_grads = True

    def __init__(self, module: nn.Module, cfg: AdamWConfig, heap, *, tp_group=None) -> None:
        self.cfg = cfg
        self.heap = heap
        self.tp_group = tp_group
        groups = bucket_groups(module)
        self.arenas = []
        for dt in (torch.bfloat16, torch.float32):
            g = [(label, [p for p in ps if p.dtype == dt]) for label, ps in groups]
            g = [(label, ps) for label, ps in g if ps]
            if g:
                self.arenas.append(_ShardedArena(g, dt, heap))
        if any(p.dtype not in (torch.bfloat16, torch.float32) for _, ps in groups for p in ps):
            raise TypeError("unsupported parameter dtype")
        self.bucket_ids = []     # global id -> (arena index, bucket index)
        self.by_label: dict = {}
        for ai, a in enumerate(self.arenas):
            for bi, (label, *_rest) in enumerate(a.buckets):
                self.by_label.setdefault(label, []).append(len(self.bucket_ids))
                self.bucket_ids.append((ai, bi))
        if len(self.bucket_ids) > _MAX_BUCKETS:
            raise ValueError(f"{len(self.bucket_ids)} gradient buckets exceed the {_MAX_BUCKETS} flag slots")
        self.n_layers = len(getattr(module, "layers", ()) or ())
        self.flags = heap.alloc(heap.size * _MAX_BUCKETS * 8)
        self._partials = torch.zeros(len(self.bucket_ids) * _PARTIALS_PER_BUCKET, dtype=torch.float32,
                                     device=heap.device)
        self._norm = torch.zeros(1, dtype=torch.float32, device=heap.device)
        self._stream = torch.cuda.Stream(device=heap.device)
        self._issued: set[int] = set()
        self._armed = False
        self._epoch = 0
        self.step_count = 0
        self._hooks = [p.register_post_accumulate_grad_hook(self._fold) for a in self.arenas for p in a.params]
        if hasattr(module, "grad_ready_callback"):
            module.grad_ready_callback = self._layer_done

    # ---------------------------------------------------------------- overlap
    def arm_overlap(self) -> None:
        """Called right before the step's last backward: buckets are reduced as their layers finish."""
        if not self._armed:
            self._epoch += 1
            self._armed = True

    def _layer_done(self, layer: int) -> None:
        if not self._armed:
            return
        labels = [layer] + (["tail"] if layer == self.n_layers - 1 else [])
        for label in labels:
            for gb in self.by_label.get(label, ()):
                self._issue(gb, overlap=True)

    def _issue(self, gb: int, *, overlap: bool) -> None:
        if gb in self._issued:
            return
        self._issued.add(gb)
        m, h = kernels(), self.heap
        ai, bi = self.bucket_ids[gb]
        a = self.arenas[ai]
        if self.tp_group is not None:
            import torch.distributed as dist

            label = a.buckets[bi][0]
            for p in a.params:
                if getattr(p, "tp_partial_grad", False) and self._label_of(a, p) == label:
                    dist.all_reduce(p.main_grad, group=self.tp_group)
        m.dp_bucket_signal(self.flags.ptrs, h.rank, _MAX_BUCKETS, gb, self._epoch)
        off, cnt, _ = a.own_range(bi, h.rank)
        parts = self._partials[gb * _PARTIALS_PER_BUCKET:(gb + 1) * _PARTIALS_PER_BUCKET]
        if overlap:
            ev = torch.cuda.Event()
            ev.record()
            with torch.cuda.stream(self._stream):
                self._stream.wait_event(ev)
                m.dp_bucket_wait(self.flags.ptrs[h.rank], h.size, _MAX_BUCKETS, gb, self._epoch, h.timeout_s)
                m.dp_reduce_scatter(a.grad_buf.ptrs, h.rank, off, cnt, 1.0 / h.size, parts)
        else:
            m.dp_bucket_wait(self.flags.ptrs[h.rank], h.size, _MAX_BUCKETS, gb, self._epoch, h.timeout_s)
            m.dp_reduce_scatter(a.grad_buf.ptrs, h.rank, off, cnt, 1.0 / h.size, parts)

    def _label_of(self, a: _ShardedArena, p) -> object:
        cache = getattr(a, "_label_cache", None)
        if cache is None:
            cache = a._label_cache = {}
            for label, off, padded, _, _ in a.buckets:
                for q, (o, _) in zip(a.params, a.param_ranges):
                    if off <= o < off + padded:
                        cache[id(q)] = label
        return cache[id(p)]

    # ---------------------------------------------------------------- update
    def step(self, *, grad_norm: Tensor | None = None) -> Tensor:
        c = self.cfg
        m = kernels()
        h = self.heap
        if not self._armed:
            self._epoch += 1
        self.step_count += 1
        b1, b2 = c.betas
        bc1 = 1.0 - b1 ** self.step_count
        bc2 = 1.0 - b2 ** self.step_count
        for gb in range(len(self.bucket_ids)):           # what the hooks did not issue
            self._issue(gb, overlap=False)
        torch.cuda.current_stream().wait_stream(self._stream)
        h.barrier(payload=self._partials)                  # norm partials -> every peer; all pulls are done
        for a in self.arenas:
            for bi in range(len(a.buckets)):
                off, cnt, lo = a.own_range(bi, h.rank)
                m.dp_adamw_allgather(a.master[lo:lo + cnt], a.m[lo:lo + cnt], a.v[lo:lo + cnt],
                                     a.main_grad[off:off + cnt], a.data_buf.ptrs, off, a.bf16, h.pad.ptrs[h.rank],
                                     float(c.grad_clip), float(c.lr), float(b1), float(b2), float(c.eps),
                                     float(c.weight_decay), float(bc1), float(bc2), self._norm)
        h.barrier()                                        # all parameter stores have landed
        self._issued.clear()
        self._armed = False
        return self._norm[0].clone()

    def grad_norm(self) -> Tensor:
        raise NotImplementedError("the sharded optimizer computes the norm inside step()")

    def state_dict(self) -> dict:
        import torch.distributed as dist

        out = []
        for a in self.arenas:
            full = {}
            for name in ("master", "m", "v"):
                parts = [torch.empty_like(a.master) for _ in range(self.heap.size)]
                dist.all_gather(parts, getattr(a, name).contiguous(), group=self.heap.group)
                full[name] = a.to_param_order(parts)
            out.append(full)
        return {"step": self.step_count, "arenas": out}

    def load_state_dict(self, sd: dict) -> None:
        self.step_count = int(sd["step"])
        for a, s in zip(self.arenas, sd["arenas"]):
            for name in ("master", "m", "v"):
                getattr(a, name).copy_(a.from_param_order(s[name].to(a.master.device).float().reshape(-1), self.heap.rank))
            src = s["master"].to(a.master.device).float().reshape(-1)
            k = 0
            for o, n in a.param_ranges:
                a.data[o:o + n].copy_(src[k:k + n].to(a.data.dtype))
                k += n
