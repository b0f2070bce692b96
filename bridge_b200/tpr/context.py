"""Per-forward TPR attention context, carried through the model in a ContextVar.

The context tells every attention layer of one model forward *what to attend
to besides itself* and collects what the layer produced:

* ``past_key_values[layer] = (K, V)`` -- the external prefix bank, packed
  ``[P_total, Hkv, D]`` (token-major, no batch dim).  With ``layout`` unset the
  forward is one segment and attends to the whole bank; with a
  :class:`SegmentBatchLayout` the forward is a packed batch of segments and
  segment ``i`` attends to ``bank[prefix_off[i] : prefix_off[i] + prefix_len[i]]``
  -- siblings point at the same span, so shared prefix KV is stored once and
  its gradient is reduced inside the attention backward.
* ``attention_backend`` -- replaces the bank when context parallelism is on.
* ``initial_gdn_states`` -- the parent's GDN conv/recurrent state per layer.
* collectors for the new post-RoPE K / raw V and the final GDN states.

Tensors are stored as given (never detached or cloned) so a prefix anchor stays
connected to the suffix's autograd graph.

Parity: verl/models/mcore/tpr/context.py:35-314 (TPRAttentionBackend protocol,
TPRAttentionContext, get/use_tpr_attention_context).  The batch layout is new:
the reference executes one segment per forward.
"""

from __future__ import annotations

from collections.abc import Iterable, Iterator, Mapping
from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass, field
from types import MappingProxyType
from typing import Any, Protocol, runtime_checkable

import torch
from torch import Tensor

KVPair = tuple[Tensor, Tensor]


def _check_layer(layer_number: int) -> None:
    if not isinstance(layer_number, int) or isinstance(layer_number, bool) or layer_number <= 0:
        raise ValueError(f"layer_number must be a positive integer, got {layer_number!r}")


def _check_kv(layer: int, k: Tensor, v: Tensor, *, length: int | None, kind: str) -> None:
    if not isinstance(k, Tensor) or not isinstance(v, Tensor):
        raise TypeError(f"layer {layer} {kind} K/V must be torch tensors")
    if k.ndim != 3 or v.ndim != 3:
        raise ValueError(
            f"layer {layer} {kind} K/V must have shape [tokens, heads, head_dim], got K={tuple(k.shape)}, "
            f"V={tuple(v.shape)}"
        )
    if k.shape[:2] != v.shape[:2]:
        raise ValueError(f"layer {layer} {kind} K/V shapes must match, got K={tuple(k.shape)}, V={tuple(v.shape)}")
    if length is not None and k.shape[0] != length:
        raise ValueError(f"layer {layer} {kind} KV sequence length must be {length}, got {k.shape[0]}")
    if k.device != v.device or k.dtype != v.dtype:
        raise ValueError(f"layer {layer} {kind} K/V device and dtype must match")


@runtime_checkable
class TPRAttentionBackend(Protocol):
    """Context-parallel attention for one segment forward."""

    @property
    def global_prefix_length(self) -> int: ...

    @property
    def global_suffix_length(self) -> int: ...

    @property
    def local_suffix_length(self) -> int: ...

    @property
    def parallel_size(self) -> int: ...

    def attention(self, layer_number: int, query: Tensor, key: Tensor, value: Tensor, *,
                  softmax_scale: float | None = None) -> Tensor: ...


@dataclass(frozen=True, slots=True)
class SegmentBatchLayout:
    """Host + device metadata of a packed batch of query segments.

    ``seq_lens[i]`` rows of segment ``i`` follow each other in the packed
    tensors; ``prefix_spans[i] = (offset, length)`` addresses the prefix bank.
    """

    seq_lens: tuple[int, ...]
    prefix_spans: tuple[tuple[int, int], ...]
    cu_seqlens: Tensor            # int32 [B+1] on the compute device
    prefix_offsets: Tensor        # int32 [B]
    prefix_lengths: Tensor        # int32 [B]
    max_seqlen: int
    max_prefix: int
    prefix_total: int
    cache: dict = field(default_factory=dict, compare=False, repr=False)

    @classmethod
    def build(cls, seq_lens, prefix_spans, *, device) -> "SegmentBatchLayout":
        seq_lens = tuple(int(n) for n in seq_lens)
        spans = tuple((int(o), int(n)) for o, n in prefix_spans)
        if len(seq_lens) != len(spans) or not seq_lens:
            raise ValueError("seq_lens and prefix_spans must be non-empty and of equal length")
        if any(n <= 0 for n in seq_lens):
            raise ValueError("every segment in a batch must be non-empty")
        if any(o < 0 or n < 0 for o, n in spans):
            raise ValueError("prefix spans must be non-negative")
        cu = [0]
        for n in seq_lens:
            cu.append(cu[-1] + n)
        meta = torch.tensor([cu, [o for o, _ in spans] + [0], [n for _, n in spans] + [0]],
                            dtype=torch.int32).to(device, non_blocking=True)
        return cls(seq_lens, spans, meta[0], meta[1, :-1], meta[2, :-1], max(seq_lens),
                   max(n for _, n in spans), max((o + n for o, n in spans), default=0))

    @property
    def batch_size(self) -> int:
        return len(self.seq_lens)

    @property
    def total_tokens(self) -> int:
        return sum(self.seq_lens)


@dataclass(slots=True)
class TPRAttentionContext:
    """External prefix state scoped to one model forward (single segment or a packed batch)."""

    prefix_length: int
    suffix_length: int
    past_key_values: Mapping[int, KVPair] = field(default_factory=dict)
    position_ids: Tensor | None = None
    attention_backend: TPRAttentionBackend | None = None
    initial_gdn_states: Mapping[int, Any] = field(default_factory=dict)
    capture_gdn_final_state: bool = True
    layout: SegmentBatchLayout | None = None
    record_new_kv: bool = True
    new_kv_observer: Any = None    # called with (key, value) as a layer records its new K/V
    _new_key_values: dict[int, KVPair] = field(default_factory=dict, init=False, repr=False)
    _new_gdn_states: dict[int, Any] = field(default_factory=dict, init=False, repr=False)

    def __post_init__(self) -> None:
        for name in ("prefix_length",):
            v = getattr(self, name)
            if not isinstance(v, int) or isinstance(v, bool) or v < 0:
                raise ValueError(f"{name} must be a non-negative integer, got {v!r}")
        if not isinstance(self.suffix_length, int) or isinstance(self.suffix_length, bool) or self.suffix_length <= 0:
            raise ValueError(f"suffix_length must be a positive integer, got {self.suffix_length!r}")
        if not isinstance(self.capture_gdn_final_state, bool):
            raise TypeError("capture_gdn_final_state must be a bool")
        if self.layout is None:
            if self.prefix_length == 0 and self.past_key_values:
                raise ValueError("past_key_values must be empty when prefix_length is 0")
            if self.prefix_length == 0 and self.initial_gdn_states:
                raise ValueError("initial_gdn_states must be empty when prefix_length is 0")
        else:
            if self.layout.total_tokens != self.suffix_length:
                raise ValueError("layout total tokens must equal suffix_length")
        if self.attention_backend is not None:
            be = self.attention_backend
            missing = [n for n in ("global_prefix_length", "global_suffix_length", "local_suffix_length",
                                   "parallel_size") if not hasattr(be, n)]
            if missing or not callable(getattr(be, "attention", None)):
                raise TypeError(f"attention_backend must implement TPRAttentionBackend; missing={missing}")
            if self.past_key_values:
                raise ValueError("past_key_values must be empty when an attention_backend is active")
            if be.global_prefix_length != self.prefix_length:
                raise ValueError("attention backend prefix length must match TPRAttentionContext")
            if be.global_suffix_length != self.suffix_length:
                raise ValueError("attention backend suffix length must match TPRAttentionContext")
            if be.local_suffix_length <= 0:
                raise ValueError("attention backend local suffix length must be positive")
        past = {}
        want = self.prefix_length if self.layout is None else None
        for layer, pair in self.past_key_values.items():
            _check_layer(layer)
            if not isinstance(pair, tuple) or len(pair) != 2:
                raise TypeError(f"layer {layer} past KV must be a (key, value) tuple")
            _check_kv(layer, pair[0], pair[1], length=want, kind="past")
            past[layer] = pair
        self.past_key_values = MappingProxyType(past)
        gdn = {}
        for layer, st in self.initial_gdn_states.items():
            _check_layer(layer)
            gdn[layer] = st
        self.initial_gdn_states = MappingProxyType(dict(sorted(gdn.items())))

    # ----------------------------------------------------------------- views
    @property
    def new_key_values(self) -> Mapping[int, KVPair]:
        return MappingProxyType(self._new_key_values)

    @property
    def new_gdn_states(self) -> Mapping[int, Any]:
        return MappingProxyType(self._new_gdn_states)

    @property
    def local_suffix_length(self) -> int:
        if self.attention_backend is None:
            return self.suffix_length
        return self.attention_backend.local_suffix_length

    # ----------------------------------------------------------------- access
    def get_past_kv(self, layer_number: int) -> KVPair | None:
        _check_layer(layer_number)
        if self.attention_backend is not None:
            raise RuntimeError("sharded attention must obtain prefix state from its attention backend")
        if self.layout is None and self.prefix_length == 0:
            return None
        if self.layout is not None and self.layout.prefix_total == 0:
            return None
        try:
            return self.past_key_values[layer_number]
        except KeyError as exc:
            raise KeyError(f"missing past KV for layer {layer_number}") from exc

    def set_new_kv(self, layer_number: int, key: Tensor, value: Tensor) -> None:
        _check_layer(layer_number)
        if self.new_kv_observer is not None:
            self.new_kv_observer((key, value))
        if not self.record_new_kv:
            return
        if layer_number in self._new_key_values:
            raise RuntimeError(f"new KV for layer {layer_number} was already recorded")
        _check_kv(layer_number, key, value, length=self.local_suffix_length, kind="new")
        self._new_key_values[layer_number] = (key, value)

    def get_initial_gdn_state(self, layer_number: int):
        _check_layer(layer_number)
        if not self.initial_gdn_states:
            if self.prefix_length == 0 or self.layout is not None:
                return None
        try:
            return self.initial_gdn_states[layer_number]
        except KeyError as exc:
            raise KeyError(f"missing initial GDN state for layer {layer_number}") from exc

    def set_new_gdn_state(self, layer_number: int, state) -> None:
        _check_layer(layer_number)
        if layer_number in self._new_gdn_states:
            raise RuntimeError(f"new GDN state for layer {layer_number} was already recorded")
        from .prefix_state import GDNLayerState

        if not isinstance(state, GDNLayerState):
            raise TypeError(f"layer {layer_number} new GDN state must be GDNLayerState")
        self._new_gdn_states[layer_number] = state

    def assert_new_kv_layers(self, expected: Iterable[int]) -> None:
        want = set(expected)
        got = set(self._new_key_values)
        if self.record_new_kv and got != want:
            raise RuntimeError(f"new KV layer mismatch: missing={sorted(want - got)}, unexpected={sorted(got - want)}")

    def assert_new_gdn_layers(self, expected: Iterable[int]) -> None:
        want = set(expected)
        got = set(self._new_gdn_states)
        if got != want:
            raise RuntimeError(f"new GDN layer mismatch: missing={sorted(want - got)}, unexpected={sorted(got - want)}")

    # ----------------------------------------------------------------- compute
    def attention(self, layer_number: int, q: Tensor, k: Tensor, v: Tensor, *, softmax_scale: float) -> Tensor:
        """Attend ``q`` to (prefix bank span | own causal K/V); records the new K/V."""
        self.set_new_kv(layer_number, k, v)
        if self.attention_backend is not None:
            return self.attention_backend.attention(layer_number, q, k, v, softmax_scale=softmax_scale)
        from ..ops.attention import tree_attention

        past = self.get_past_kv(layer_number)
        if self.layout is None:
            n = q.shape[0]
            layout = _single_layout(n, self.prefix_length if past is not None else 0, q.device)
        else:
            layout = self.layout
        pk, pv = past if past is not None else (None, None)
        return tree_attention(q, k, v, pk, pv, layout, softmax_scale=softmax_scale)


_LAYOUT_CACHE: dict[tuple, SegmentBatchLayout] = {}


def _single_layout(n: int, prefix: int, device) -> SegmentBatchLayout:
    key = (n, prefix, str(device))
    lay = _LAYOUT_CACHE.get(key)
    if lay is None:
        if len(_LAYOUT_CACHE) > 256:
            _LAYOUT_CACHE.clear()
        lay = _LAYOUT_CACHE[key] = SegmentBatchLayout.build((n,), ((0, prefix),), device=device)
    return lay


_ACTIVE: ContextVar[TPRAttentionContext | None] = ContextVar("tpr_attention_context", default=None)


def get_tpr_attention_context() -> TPRAttentionContext | None:
    return _ACTIVE.get()


@contextmanager
def use_tpr_attention_context(context: TPRAttentionContext) -> Iterator[TPRAttentionContext]:
    if not isinstance(context, TPRAttentionContext):
        raise TypeError(f"context must be a TPRAttentionContext, got {type(context).__name__}")
    token = _ACTIVE.set(context)
    try:
        yield context
    finally:
        _ACTIVE.reset(token)
