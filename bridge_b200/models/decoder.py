"""Decoder-only policy model (Qwen3 dense / hybrid GDN / hybrid MoE).

``forward(input_ids [T], position_ids [T]) -> hidden [T, hidden]`` runs the
embedding, every decoder layer (attention layers read the active TPR context)
and the final RMSNorm on a packed token stream.  The LM head is applied only
to the rows that carry a loss term, through
:func:`~bridge_b200.ops.logprob.fused_lm_head_logprob` (PPO) or
:meth:`logits` (CE / debugging) -- the full ``[T, vocab]`` logits of prompt
rows are never computed.
"""

from __future__ import annotations

import functools

import torch
import torch.nn as nn
from torch import Tensor

from ..ops.norm import add_rmsnorm
from ..parallel.tp import (VocabParallelEmbedding, copy_to_tp, gather_from_sp, reduce_scatter_to_sp, tp_rank,
                           tp_size)
from .config import ModelConfig
from .layers import DecoderLayer, RMSNorm, RotaryEmbedding


def _layer_done_hook(callback, layer: int, grad):
    callback(layer)


class DecoderModel(nn.Module):
    def __init__(self, cfg: ModelConfig, *, tp_group=None, sequence_parallel: bool = False, ep_group=None,
                 device=None) -> None:
        super().__init__()
        self.config = cfg
        self.tp_group = tp_group
        self.sequence_parallel = sequence_parallel and tp_size(tp_group) > 1
        self.embed_tokens = VocabParallelEmbedding(cfg.vocab_size, cfg.hidden_size, group=tp_group,
                                                   std=cfg.init_std, device=device)
        self.layers = nn.ModuleList(
            DecoderLayer(cfg, i + 1, tp_group=tp_group, sequence_parallel=self.sequence_parallel,
                         ep_group=ep_group, device=device)
            for i in range(cfg.num_layers)
        )
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_eps, device=device)
        if self.sequence_parallel:  # norms see only this rank's token shard: gradients summed over TP
            for layer in self.layers:
                layer.input_layernorm.weight.tp_partial_grad = True  # type: ignore[attr-defined]
                layer.post_attention_layernorm.weight.tp_partial_grad = True  # type: ignore[attr-defined]
            self.norm.weight.tp_partial_grad = True  # type: ignore[attr-defined]

        self.rotary_pos_emb = RotaryEmbedding(cfg.head_dim, cfg.rope_theta)
        if cfg.tie_word_embeddings:
            self.lm_head = None
        else:
            n = tp_size(tp_group)
            self.lm_head = nn.Parameter(torch.randn(cfg.vocab_size // n, cfg.hidden_size, device=device,
                                                    dtype=torch.bfloat16) * cfg.init_std)
            self.lm_head.tp_split_dim = 0  # type: ignore[attr-defined]
        self.vocab_size = cfg.vocab_size
        # Called with a layer index when the backward has finished that layer (its input gradient is
        # computed); the sharded data-parallel optimizer uses it to start reducing the layer's bucket.
        self.grad_ready_callback = None

    # ------------------------------------------------------------------ metadata
    @property
    def attention_layer_numbers(self) -> tuple[int, ...]:
        return self.config.attention_layer_numbers

    @property
    def gdn_layer_numbers(self) -> tuple[int, ...]:
        return self.config.gdn_layer_numbers

    @property
    def head_weight(self) -> Tensor:
        return self.embed_tokens.weight if self.lm_head is None else self.lm_head

    @property
    def vocab_start(self) -> int:
        return tp_rank(self.tp_group) * (self.vocab_size // tp_size(self.tp_group))

    # ------------------------------------------------------------------ compute
    def forward(self, input_ids: Tensor, position_ids: Tensor, max_position: int | None = None) -> Tensor:
        if input_ids.ndim == 2:  # [1, T] accepted for single-sequence callers
            input_ids, position_ids = input_ids[0], position_ids[0]
        rope = self.rotary_pos_emb(position_ids, max_position)
        if self.sequence_parallel:
            if input_ids.shape[0] % tp_size(self.tp_group):
                raise ValueError("sequence-parallel segments must be divisible by the TP size")
            # vocab-sharded partial rows -> reduce-scatter over tokens (backward: all-gather, so every
            # rank's vocab shard sees the gradient of every token)
            x = reduce_scatter_to_sp(self.embed_tokens(input_ids, reduce=False), self.tp_group)
        else:
            x = self.embed_tokens(input_ids)
        pending = None      # each block's MLP output is added inside the next block's first norm
        cb = self.grad_ready_callback
        for i, layer in enumerate(self.layers):
            if cb is not None and x.requires_grad:
                x.register_hook(functools.partial(_layer_done_hook, cb, i))
            x, pending = layer(x, rope, pending, True)
        x = self.norm(x) if pending is None else add_rmsnorm(x, pending, self.norm.weight, self.norm.eps)[1]
        if self.sequence_parallel:
            x = gather_from_sp(x, self.tp_group)
        return x

    def head_input(self, hidden_rows: Tensor) -> Tensor:
        """Prepare selected hidden rows for the (vocab-parallel) LM head.

        Each TP rank's head backward yields a partial ``dh`` (its vocab shard).  Without sequence
        parallelism they are summed here (all-reduce); with it the final hidden states came out of
        :func:`gather_from_sp`, whose backward reduce-scatter already sums them -- summing here too
        would count every contribution TP times."""
        return hidden_rows if self.sequence_parallel else copy_to_tp(hidden_rows, self.tp_group)

    def logits(self, hidden_rows: Tensor) -> Tensor:
        """Local-vocab logits ``[U, V/TP]`` of selected rows."""
        from ..ops.gemm import linear

        return linear(self.head_input(hidden_rows), self.head_weight)


def build_model(cfg: ModelConfig, *, device=None, seed: int = 0, tp_group=None, sequence_parallel=False,
                ep_group=None, dtype: torch.dtype | None = None) -> DecoderModel:
    """Random-init model; every rank of a TP group uses a rank-dependent stream for its shard.

    Parameters are created on the host (deterministic across devices) and then
    moved; ``dtype`` (e.g. FP32 for CPU oracles) converts every parameter.
    """
    g_state = torch.random.get_rng_state()
    dev = torch.device(device) if device is not None else torch.device("cpu")
    cuda_state = torch.cuda.get_rng_state(dev) if dev.type == "cuda" else None
    torch.manual_seed(seed * 7919 + 104729 * tp_rank(tp_group))
    try:
        # Large models initialise directly on the GPU; host init is used for CPU runs.
        model = DecoderModel(cfg, tp_group=tp_group, sequence_parallel=sequence_parallel, ep_group=ep_group,
                             device=dev)
    finally:
        torch.random.set_rng_state(g_state)
        if cuda_state is not None:
            torch.cuda.set_rng_state(cuda_state, dev)
    if dtype is not None:
        model = model.to(dtype)
    return model
