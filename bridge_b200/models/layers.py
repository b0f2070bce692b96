"""Decoder layers: TPR-aware self-attention, Gated DeltaNet, SwiGLU MLP and MoE.

All layers take packed token-major activations ``[T, hidden]`` and read the
active :class:`~bridge_b200.tpr.context.TPRAttentionContext` (if any) to find
their external prefix: attention layers attend to the prefix KV bank (or the
CP backend), GDN layers start from the parent's conv/recurrent state.

Parity: verl/models/mcore/tpr/attention.py:44-176 (TPRSelfAttention: QKV,
qk-norm, RoPE, prefix attention, output gate, new-KV collection) and
verl/models/mcore/tpr/gated_delta_net.py:75-263 (TPRGatedDeltaNet stateful
conv + delta rule + gated norm).  The modules are this framework's own
(no Megatron/MindSpeed base classes).
"""

from __future__ import annotations

import math

import torch
import torch.nn as nn
from torch import Tensor

from ..ops.activation import swiglu
from ..ops.attention import tree_attention
from ..ops.gdn import causal_conv1d, chunk_gated_delta_rule, gated_rmsnorm, gdn_gates, l2norm
from ..ops.norm import add_rmsnorm, qk_norm_rope, rmsnorm, rope_cos_sin
from ..parallel.tp import ColumnParallelLinear, RowParallelLinear, tp_size, scaled_init_std
from ..tpr.context import get_tpr_attention_context, _single_layout
from .config import ModelConfig


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6, dtype=torch.bfloat16, device=None) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, dtype=dtype, device=device))

    def forward(self, x: Tensor) -> Tensor:
        return rmsnorm(x, self.weight, self.eps)


class RotaryEmbedding(nn.Module):
    """Maps absolute positions to FP32 ``(cos, sin) [T, head_dim/2]`` (cached per device)."""

    def __init__(self, head_dim: int, theta: float) -> None:
        super().__init__()
        self.head_dim, self.theta = head_dim, theta
        self.cp_group = None
        self._table: dict[str, tuple[Tensor, Tensor]] = {}

    def table(self, device, max_pos: int) -> tuple[Tensor, Tensor]:
        key = str(device)
        t = self._table.get(key)
        if t is None or t[0].shape[0] < max_pos:
            n = max(max_pos, 4096)
            n = 1 << (n - 1).bit_length()
            t = rope_cos_sin(torch.arange(n, device=device), self.head_dim, self.theta)
            self._table[key] = t
        return t

    def forward(self, positions: Tensor, max_position: int | None = None) -> tuple[Tensor, Tensor]:
        if max_position is None:  # host sync; executors pass the bound they already know
            max_position = int(positions.max().item()) if positions.numel() else 0
        cos, sin = self.table(positions.device, max_position + 1)
        return cos.index_select(0, positions), sin.index_select(0, positions)


class TPRSelfAttention(nn.Module):
    """GQA self-attention with qk-RMSNorm, RoPE and an optional sigmoid output gate."""

    tpr_state_kind = "kv"

    def __init__(self, cfg: ModelConfig, layer_number: int, *, tp_group=None, sequence_parallel=False,
                 device=None) -> None:
        super().__init__()
        n = tp_size(tp_group)
        if cfg.num_heads % n or cfg.num_kv_heads % n:
            raise ValueError("attention heads must divide evenly over the TP group")
        self.layer_number = layer_number
        self.hq, self.hkv, self.d = cfg.num_heads // n, cfg.num_kv_heads // n, cfg.head_dim
        self.gate = cfg.attention_output_gate
        q_out = cfg.num_heads * cfg.head_dim * (2 if self.gate else 1)
        # Fused QKV weight, TP-sharded per rank as [q(+gate) | k | v] of the local heads.
        self.qkv = ColumnParallelLinear(cfg.hidden_size, q_out + 2 * cfg.num_kv_heads * cfg.head_dim,
                                        group=tp_group, sequence_parallel=sequence_parallel, std=cfg.init_std,
                                        device=device)
        self.o_proj = RowParallelLinear(cfg.num_heads * cfg.head_dim, cfg.hidden_size, group=tp_group,
                                        sequence_parallel=sequence_parallel,
                                        std=scaled_init_std(cfg.init_std, cfg.num_layers), device=device)
        self.q_norm = RMSNorm(cfg.head_dim, cfg.rms_eps, device=device) if cfg.qk_norm else None
        self.k_norm = RMSNorm(cfg.head_dim, cfg.rms_eps, device=device) if cfg.qk_norm else None
        if n > 1:  # replicated weights that only see this rank's heads: gradients are summed over TP
            for norm in (self.q_norm, self.k_norm):
                if norm is not None:
                    norm.weight.tp_partial_grad = True  # type: ignore[attr-defined]
        self.eps = cfg.rms_eps
        self.scale = 1.0 / math.sqrt(cfg.head_dim)

    def forward(self, x: Tensor, rope: tuple[Tensor, Tensor]) -> Tensor:
        qkv = self.qkv(x)
        t = qkv.shape[0]
        qd = self.hq * self.d * (2 if self.gate else 1)
        kd = self.hkv * self.d
        q_all, k, v = qkv.split((qd, kd, kd), dim=-1)
        if self.gate:
            q_all = q_all.view(t, self.hq, 2 * self.d)
            q, gate = q_all[..., : self.d], q_all[..., self.d:]
        else:
            q, gate = q_all.view(t, self.hq, self.d), None
        k = k.view(t, self.hkv, self.d)
        v = v.view(t, self.hkv, self.d)
        cos, sin = rope
        q, k = qk_norm_rope(q, k, self.q_norm.weight if self.q_norm is not None else None,
                            self.k_norm.weight if self.k_norm is not None else None, cos, sin, self.eps)
        v = v.contiguous()
        ctx = get_tpr_attention_context()
        if ctx is None:
            o = tree_attention(q, k, v, None, None, _single_layout(t, 0, q.device), softmax_scale=self.scale)
        else:
            o = ctx.attention(self.layer_number, q, k, v, softmax_scale=self.scale)
        if gate is not None:
            o = o * torch.sigmoid(gate.float()).to(o.dtype)
        return self.o_proj(o.reshape(t, self.hq * self.d))


class TPRGatedDeltaNet(nn.Module):
    """Qwen3-Next style Gated DeltaNet with stateful conv and recurrent continuation."""

    tpr_state_kind = "gdn"

    def __init__(self, cfg: ModelConfig, layer_number: int, *, tp_group=None, sequence_parallel=False,
                 device=None) -> None:
        super().__init__()
        n = tp_size(tp_group)
        if cfg.gdn_num_qk_heads % n or cfg.gdn_num_v_heads % n:
            raise ValueError("GDN heads must divide evenly over the TP group")
        self.layer_number = layer_number
        self.hk, self.hv, self.dk = cfg.gdn_num_qk_heads // n, cfg.gdn_num_v_heads // n, cfg.gdn_head_dim
        self.dv = cfg.gdn_head_dim
        self.w = cfg.gdn_conv_kernel
        self.chunk = cfg.gdn_chunk_size
        kd, vd = cfg.gdn_num_qk_heads * self.dk, cfg.gdn_num_v_heads * self.dv
        # under sequence parallelism the input projection all-gathers the token shard first (and the output
        # projection reduce-scatters), so the conv and the delta rule always see whole sequences
        self.in_proj = ColumnParallelLinear(cfg.hidden_size, 2 * kd + 2 * vd + 2 * cfg.gdn_num_v_heads,
                                            group=tp_group, sequence_parallel=sequence_parallel, std=cfg.init_std,
                                            device=device)
        c_local = (2 * kd + vd) // n
        self.conv_weight = nn.Parameter(torch.randn(c_local, self.w, device=device, dtype=torch.bfloat16)
                                        * (1.0 / math.sqrt(self.w)))
        self.A_log = nn.Parameter(torch.log(torch.empty(self.hv, device=device).uniform_(1, 16)))
        self.dt_bias = nn.Parameter(torch.zeros(self.hv, device=device))
        self.norm_weight = nn.Parameter(torch.ones(self.dv, device=device, dtype=torch.bfloat16))
        if n > 1:  # shared across heads; each TP rank sees only its heads
            self.norm_weight.tp_partial_grad = True  # type: ignore[attr-defined]
        self.out_proj = RowParallelLinear(vd, cfg.hidden_size, group=tp_group, sequence_parallel=sequence_parallel,
                                          std=scaled_init_std(cfg.init_std, cfg.num_layers), device=device)
        self.eps = cfg.rms_eps
        self.scale = 1.0 / math.sqrt(self.dk)

    @property
    def conv_channels(self) -> int:
        return self.conv_weight.shape[0]

    def forward(self, x: Tensor, rope=None) -> Tensor:
        from ..tpr.prefix_state import GDNLayerState

        t = x.shape[0]
        kd, vd = self.hk * self.dk, self.hv * self.dv
        ctx = get_tpr_attention_context()
        backend = getattr(ctx, "attention_backend", None) if ctx is not None else None
        cp_group = getattr(backend, "cp_group", None)
        if cp_group is not None and torch.distributed.get_world_size(cp_group) > 1:
            from ..parallel.gdn_state import forward_gdn_cp_tpr

            return forward_gdn_cp_tpr(self, x, ctx, backend)          # CP-sharded tokens: head-parallel
        proj = self.in_proj(x)                 # all tokens of the forward (gathered under SP)
        t = proj.shape[0]
        qkv, z, b, a = proj.split((2 * kd + vd, vd, self.hv, self.hv), dim=-1)
        if ctx is not None and ctx.layout is not None:
            cu = [0]
            for n in ctx.layout.seq_lens:
                cu.append(cu[-1] + n)
            cu_dev = ctx.layout.cu_seqlens
        else:
            cu, cu_dev = [0, t], None
        nseq = len(cu) - 1
        init = ctx.get_initial_gdn_state(self.layer_number) if ctx is not None else None
        h_conv = h_rec = None
        if init is not None:
            h_conv, h_rec = init.conv_state, init.recurrent_state
            if h_conv.shape[0] == 1 and nseq > 1:
                h_conv = h_conv.expand(nseq, -1, -1)
                h_rec = h_rec.expand(nseq, -1, -1, -1)
        y, conv_final = causal_conv1d(qkv, self.conv_weight, None, cu, cu_dev, h_conv, activation=True)
        q, k, v = y.split((kd, kd, vd), dim=-1)
        q = l2norm(q.reshape(t, self.hk, self.dk))
        k = l2norm(k.reshape(t, self.hk, self.dk))
        v = v.reshape(t, self.hv, self.dv)
        rep = self.hv // self.hk
        if rep > 1:
            q = q.repeat_interleave(rep, dim=1)
            k = k.repeat_interleave(rep, dim=1)
        g, beta = gdn_gates(a, b, self.A_log, self.dt_bias)
        o, rec_final = chunk_gated_delta_rule(q, k, v, g, beta, cu, cu_dev, h_rec, scale=self.scale,
                                              chunk_size=self.chunk)
        if ctx is not None and ctx.capture_gdn_final_state:
            ctx.set_new_gdn_state(self.layer_number, GDNLayerState(conv_final, rec_final))
        o = gated_rmsnorm(o, z.reshape(t, self.hv, self.dv), self.norm_weight, self.eps)
        return self.out_proj(o.reshape(t, vd))


class SwiGLUMLP(nn.Module):
    def __init__(self, hidden: int, ffn: int, *, tp_group=None, sequence_parallel=False, std=0.02,
                 out_std=0.02, device=None) -> None:
        super().__init__()
        n = tp_size(tp_group)
        if ffn % n:
            raise ValueError("FFN size must divide evenly over the TP group")
        # FC1 holds [local gate | local up] per rank.
        self.fc1 = ColumnParallelLinear(hidden, 2 * ffn, group=tp_group, sequence_parallel=sequence_parallel,
                                        std=std, device=device)
        self.fc2 = RowParallelLinear(ffn, hidden, group=tp_group, sequence_parallel=sequence_parallel, std=out_std,
                                     device=device)

    def forward(self, x: Tensor) -> Tensor:
        return self.fc2(swiglu(self.fc1(x)))


class DecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig, layer_number: int, *, tp_group=None, sequence_parallel=False,
                 ep_group=None, device=None) -> None:
        super().__init__()
        kind = cfg.types[layer_number - 1]
        self.layer_number = layer_number
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_eps, device=device)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_eps, device=device)
        if kind == "attention":
            self.self_attention = TPRSelfAttention(cfg, layer_number, tp_group=tp_group,
                                                   sequence_parallel=sequence_parallel, device=device)
        else:
            self.self_attention = TPRGatedDeltaNet(cfg, layer_number, tp_group=tp_group,
                                                   sequence_parallel=sequence_parallel, device=device)
        if cfg.is_moe:
            from .moe import MoELayer

            self.mlp = MoELayer(cfg, ep_group=ep_group, device=device)
        else:
            self.mlp = SwiGLUMLP(cfg.hidden_size, cfg.intermediate_size, tp_group=tp_group,
                                 sequence_parallel=sequence_parallel, std=cfg.init_std,
                                 out_std=scaled_init_std(cfg.init_std, cfg.num_layers), device=device)

    def forward(self, x: Tensor, rope, pending: Tensor | None = None, defer_residual: bool = False):
        """Pre-norm block ``x + attn(norm1(x))`` then ``+ mlp(norm2(.))``.

        Each residual add is fused into the RMSNorm that reads its result.  With ``pending`` (the
        previous block's MLP output, not yet added) the block computes ``x + pending`` inside its
        first norm; with ``defer_residual`` it returns ``(h, mlp_out)`` and leaves the last add to
        the next block (or the final norm) instead of returning ``h + mlp_out``."""
        ln1, ln2 = self.input_layernorm, self.post_attention_layernorm
        if pending is None:
            y = ln1(x)
        else:
            x, y = add_rmsnorm(x, pending, ln1.weight, ln1.eps)
        h, y = add_rmsnorm(x, self.self_attention(y, rope), ln2.weight, ln2.eps)
        out = self.mlp(y)
        return (h, out) if defer_residual else h + out
