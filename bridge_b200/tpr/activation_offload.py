"""Activation offload to pinned host memory, scoped to one Pop / VisitLeaf.

While the scope is active, every tensor autograd saves (above ``min_bytes``)
is copied device->host on a side stream right after it is produced; the
device copy is released as soon as the D2H completes.  When the backward of
decoder layer ``L`` starts, the saved tensors of layer ``L-1`` are copied back
host->device on a second stream (prefetch), so the H2D of one layer overlaps
the backward math of the next.  The prefix-KV anchors of the segment (and the
new K/V a Pop hands to autograd as roots) are never offloaded: they are read
by every descendant and must stay resident.

Pinned host memory comes in large slabs shared by every scope: a scope packs
its tensors first-fit into the slabs it holds and returns them all at its
release, so chunks of any token count reuse the same host memory and
steady-state steps do no ``cudaHostAlloc``.

Parity: verl/models/mcore/tpr/activation_offload.py:61-328 (scope, limits,
protected external storages, forced same-layer restore).  Built on
``torch.autograd.graph.saved_tensors_hooks`` + ``cudaMemcpyAsync`` on
dedicated streams instead of MindSpeed SwapPrefetch.
"""

from __future__ import annotations

import functools
import os
from dataclasses import dataclass, field

import torch
from torch import Tensor, nn


def _env_min_bytes() -> int:
    return int(os.environ.get("TPR_OFFLOAD_MIN_BYTES", str(1 << 20)))


def _env_inflight_bytes() -> int:
    return int(os.environ.get("TPR_OFFLOAD_INFLIGHT_BYTES", str(16 << 30)))


@dataclass(frozen=True)
class OffloadConfig:
    enabled: bool = False
    min_bytes: int = field(default_factory=_env_min_bytes)     # smaller saved tensors stay on the device
    # device bytes whose device->host copy may still be pending: above it the forward waits for the
    # oldest copies (the host link is slower than the GPU produces activations, and a tensor's device
    # memory is only released once its copy finished)
    max_inflight_bytes: int = field(default_factory=_env_inflight_bytes)
    prefetch: bool = True
    force_restore_sync: bool = os.environ.get("TPR_OFFLOAD_B_FORCE_RESTORE_SYNC", "0") == "1"


def validate_activation_offload(model: nn.Module, cp_size: int, cp_backend, cfg: OffloadConfig | None) -> None:
    """Offload supports CP1 and the ring backend (any CP size); other backends are rejected."""
    if cfg is None or not cfg.enabled:
        return
    name = getattr(cp_backend, "backend_name", None)
    if cp_size > 1 and name != "ring":
        raise NotImplementedError(f"activation offload requires CP=1 or the ring backend, got {name!r}")


def _env_slab_bytes() -> int:
    return int(os.environ.get("TPR_OFFLOAD_SLAB_BYTES", str(1 << 30)))


_ALIGN = 512


class _PinnedSlabs:
    """Free pinned host slabs (uint8).  Tensors of every shape and dtype are packed into them, so the
    host memory held is the peak of bytes offloaded at once (plus the unused slab tails), not one buffer
    per distinct tensor size: chunks differ in token count, and a pool keyed by exact size would pin a
    fresh set of buffers for every chunk shape."""

    def __init__(self) -> None:
        self.free: list[Tensor] = []

    def take(self, nbytes: int) -> Tensor:
        fits = [s for s in self.free if s.numel() >= nbytes]
        if fits:
            slab = min(fits, key=lambda s: s.numel())
            self.free.remove(slab)
            return slab
        unit = _env_slab_bytes()
        size = max(unit, -(-nbytes // unit) * unit)
        return torch.empty(size, dtype=torch.uint8, pin_memory=torch.cuda.is_available())

    def give(self, slab: Tensor) -> None:
        self.free.append(slab)

    def held_bytes(self) -> int:
        return sum(s.numel() for s in self.free)


_SLABS = _PinnedSlabs()


class _HostArena:
    """The slabs one offload scope holds, filled first-fit."""

    def __init__(self) -> None:
        self.slabs: list[list] = []          # [slab, bytes used]

    def alloc(self, numel: int, dtype) -> Tensor:
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        need = -(-nbytes // _ALIGN) * _ALIGN
        for entry in self.slabs:
            slab, used = entry
            if slab.numel() - used >= need:
                entry[1] = used + need
                return slab[used:used + nbytes].view(dtype)
        slab = _SLABS.take(need)
        self.slabs.append([slab, need])
        return slab[:nbytes].view(dtype)

    def release(self) -> None:
        for slab, _ in self.slabs:
            _SLABS.give(slab)
        self.slabs.clear()


class _Saved:
    __slots__ = ("host", "shape", "dtype", "device", "d2h_done", "layer", "restored", "h2d_done")

    def __init__(self, host, shape, dtype, device, d2h_done, layer):
        self.host, self.shape, self.dtype, self.device = host, shape, dtype, device
        self.d2h_done, self.layer = d2h_done, layer
        self.restored: Tensor | None = None
        self.h2d_done = None


class ActivationOffloader:
    """saved_tensors_hooks pair plus per-layer prefetch bookkeeping."""

    def __init__(self, cfg: OffloadConfig, protected: list[Tensor] | tuple = ()) -> None:
        self.cfg = cfg
        self.protected = {t.untyped_storage().data_ptr() for t in protected if isinstance(t, Tensor)}
        self.layer = -1
        self.by_layer: dict[int, list[_Saved]] = {}
        self.cuda = torch.cuda.is_available()
        self.d2h = torch.cuda.Stream() if self.cuda else None
        self.h2d = torch.cuda.Stream() if self.cuda else None
        self.offloaded_bytes = 0
        self._inflight: list = []          # (d2h done event, bytes), oldest first
        self._inflight_bytes = 0
        self.arena = _HostArena()

    def protect(self, tensors) -> None:
        for t in tensors:
            if isinstance(t, Tensor):
                self.protected.add(t.untyped_storage().data_ptr())

    # -- hooks
    def pack(self, t: Tensor):
        nbytes = t.numel() * t.element_size()
        if (nbytes < self.cfg.min_bytes or isinstance(t, nn.Parameter) or t.untyped_storage().data_ptr()
                in self.protected or not t.is_contiguous()):
            return t
        host = self.arena.alloc(t.numel(), t.dtype)
        if t.is_cuda:
            ev = torch.cuda.Event()
            ev.record()
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(ev)
                host.copy_(t.reshape(-1), non_blocking=True)
                t.record_stream(self.d2h)
                done = torch.cuda.Event()
                done.record()
            self._inflight.append((done, nbytes))
            self._inflight_bytes += nbytes
            while self._inflight_bytes > self.cfg.max_inflight_bytes and len(self._inflight) > 1:
                old_ev, old_n = self._inflight.pop(0)
                old_ev.synchronize()
                self._inflight_bytes -= old_n
        else:
            host.copy_(t.reshape(-1))
            done = None
        s = _Saved(host, t.shape, t.dtype, t.device, done, self.layer)
        self.by_layer.setdefault(self.layer, []).append(s)
        self.offloaded_bytes += nbytes
        return s

    def _restore(self, s: _Saved, stream=None) -> None:
        if s.restored is not None:
            return
        if s.device.type == "cuda":
            # allocate from the compute stream's pool (the tensor is consumed there; a prefetch-stream pool
            # would hold its own copies of freed blocks), fill it on the prefetch stream
            main = torch.cuda.current_stream()
            dev = torch.empty(s.shape, dtype=s.dtype, device=s.device)
            copy_stream = stream if stream is not None else main
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(s.d2h_done)
                if copy_stream is not main:
                    # the block may have been freed by compute work still in flight: write after it
                    copy_stream.wait_stream(main)
                dev.view(-1).copy_(s.host, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record()
            if copy_stream is not main:
                dev.record_stream(copy_stream)
            s.restored, s.h2d_done = dev, ev
        else:
            s.restored = s.host.view(s.shape).clone()

    def unpack(self, s):
        if isinstance(s, Tensor):
            return s
        if s.restored is None:
            self._restore(s)
        if s.h2d_done is not None:
            torch.cuda.current_stream().wait_event(s.h2d_done)
            if self.cfg.force_restore_sync:
                s.h2d_done.synchronize()
            s.restored.record_stream(torch.cuda.current_stream())
        out = s.restored
        # the consumer owns the restored tensor now: keeping a reference here (``by_layer`` lives until
        # release) would hold every restored activation on the device until the scope ends
        s.restored, s.h2d_done = None, None
        return out

    def prefetch_layer(self, layer: int) -> None:
        if not self.cfg.prefetch:
            return
        for s in self.by_layer.get(layer, ()):
            self._restore(s, self.h2d)

    def release(self) -> None:
        """Return the pinned slabs once no copy can still touch them: the D2H copies have finished,
        and so has every H2D prefetch (one that was issued but never unpacked may still be reading
        its host buffer)."""
        if self.cuda:
            torch.cuda.current_stream().wait_stream(self.d2h)
            torch.cuda.current_stream().wait_stream(self.h2d)
            self.d2h.synchronize()
            self.h2d.synchronize()
        self.by_layer.clear()
        self.arena.release()


class _LayerTracker:
    """Forward pre-hooks record the current layer; backward pre-hooks prefetch the layer below."""

    def __init__(self, model: nn.Module, off: ActivationOffloader) -> None:
        self.handles = []
        layers = getattr(model, "layers", None)
        if layers is None:
            return
        for i, layer in enumerate(layers):
            self.handles.append(layer.register_forward_pre_hook(functools.partial(self._enter, off, i)))
            self.handles.append(layer.register_full_backward_pre_hook(functools.partial(self._bwd, off, i)))

    @staticmethod
    def _enter(off, i, module, args):
        off.layer = i

    @staticmethod
    def _bwd(off, i, module, grad_output):
        off.prefetch_layer(i - 1)

    def remove(self) -> None:
        for h in self.handles:
            h.remove()


class DeferredOffload:
    """Offload for a forward whose backward runs later (the forest executor's retained push chunks).

    ``capture()`` wraps the forward (saved tensors go to host as they are produced); ``backward()``
    wraps the later backward (layer-ahead prefetch hooks) and releases the pinned buffers after it."""

    def __init__(self, model: nn.Module, cfg: OffloadConfig, protected=()) -> None:
        self.model = model
        self.off = ActivationOffloader(cfg, protected)

    def capture(self):
        import contextlib

        @contextlib.contextmanager
        def scope():
            tracker = _ForwardTracker(self.model, self.off)
            try:
                with torch.autograd.graph.saved_tensors_hooks(self.off.pack, self.off.unpack):
                    yield self.off
            finally:
                tracker.remove()

        return scope()

    def backward(self):
        import contextlib

        @contextlib.contextmanager
        def scope():
            tracker = _LayerTracker(self.model, self.off)
            try:
                yield self.off
            finally:
                tracker.remove()
                self.off.release()

        return scope()


class _ForwardTracker(_LayerTracker):
    """Only the forward pre-hooks (layer bookkeeping for the later prefetch)."""

    def __init__(self, model: nn.Module, off: ActivationOffloader) -> None:
        self.handles = []
        for i, layer in enumerate(getattr(model, "layers", ()) or ()):
            self.handles.append(layer.register_forward_pre_hook(functools.partial(self._enter, off, i)))


def offload_scope(model: nn.Module, cfg: OffloadConfig, protected=()):
    """Context manager installing the offload hooks for one segment execution."""
    import contextlib

    @contextlib.contextmanager
    def scope():
        off = ActivationOffloader(cfg, protected)
        tracker = _LayerTracker(model, off)
        try:
            with torch.autograd.graph.saved_tensors_hooks(off.pack, off.unpack):
                yield off
        finally:
            tracker.remove()
            off.release()

    return scope()


def with_activation_offload(method):
    """Decorator for executor methods: runs them inside an offload scope when enabled."""

    @functools.wraps(method)
    def wrapper(self, *args, **kwargs):
        cfg = getattr(self, "activation_offload", None)
        if cfg is None or not cfg.enabled:
            return method(self, *args, **kwargs)
        protected = []
        for e in getattr(self, "kv_stack", ()).entries() if hasattr(getattr(self, "kv_stack", None), "entries") else ():
            for k, v in e.state.key_values.values():
                protected += [k, v]
        with offload_scope(self.model, cfg, protected):
            return method(self, *args, **kwargs)

    return wrapper
