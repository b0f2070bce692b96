"""Checkpoints: HF-format safetensors weights (TP-sharded load/save) and resumable optimizer state.

Weights use the Hugging Face Qwen3 / Qwen3-Next tensor names, so a checkpoint
written here loads in HF and vice versa:

* ``model.embed_tokens.weight`` (vocab-sharded over TP), ``model.norm.weight``,
  ``lm_head.weight`` when untied;
* attention: ``self_attn.{q,k,v,o}_proj.weight``, ``self_attn.{q,k}_norm.weight``
  -- this framework's fused per-rank QKV rows are ``[q(+gate) | k | v]`` of the
  rank's heads (heads split evenly over TP), ``o_proj`` is column-split;
* MLP: ``mlp.{gate,up,down}_proj.weight`` -- fused FC1 rows are
  ``[gate_local | up_local]``, ``down_proj`` column-split;
* MoE: ``mlp.gate.weight`` (router), ``mlp.experts.{e}.{gate,up,down}_proj.weight``,
  ``mlp.shared_expert.{gate,up,down}_proj.weight``, ``mlp.shared_expert_gate.weight``;
* GDN layers: ``linear_attn.in_proj.weight`` (rows ``[q|k|v|z|b|a]``), ``linear_attn.conv1d.weight``
  (``[C, 1, W]``, channels ``[q|k|v]``), ``linear_attn.{A_log,dt_bias,norm.weight,out_proj.weight}``;
  under TP every rank holds its heads' slice of each section, in the same section order.

Optimizer state is saved per rank (``optim_rank{r}.pt``: FP32 master, Adam
moments, step) next to ``model.safetensors`` and a ``meta.json`` with the step
counter, so training resumes exactly.

Parity: the reference defines no checkpoint format of its own and loads HF
Qwen3 safetensors with this TP mapping
(tests/models/mcore/tpr/parallel/_qwen3_tp_checkpoint.py:108-211).
"""

from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist
from torch import Tensor

from ..parallel.tp import tp_rank, tp_size


def _split(t: Tensor, dim: int, group) -> Tensor:
    return t.chunk(tp_size(group), dim=dim)[tp_rank(group)].contiguous()


def _gather(t: Tensor, dim: int, group) -> Tensor:
    if tp_size(group) == 1:
        return t
    parts = [torch.empty_like(t) for _ in range(tp_size(group))]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.cat(parts, dim=dim)


def _split_sections(t: Tensor, sizes: list[int], group) -> Tensor:
    """Rank's slice of every section of dim 0 (global section sizes ``sizes``), concatenated."""
    if tp_size(group) == 1:
        return t
    return torch.cat([s_.chunk(tp_size(group), 0)[tp_rank(group)] for s_ in t.split(sizes, 0)], 0).contiguous()


def _gather_sections(t: Tensor, sizes_local: list[int], group) -> Tensor:
    """Inverse of :func:`_split_sections`: every section gathered over TP, sections concatenated."""
    if tp_size(group) == 1:
        return t
    return torch.cat([_gather(s_, 0, group) for s_ in t.split(sizes_local, 0)], 0)


def _gdn_sections(cfg, n: int) -> tuple[list[int], list[int]]:
    """Global row sections of the GDN input projection ``[q|k|v|z|b|a]`` and conv channels ``[q|k|v]``
    (each rank holds its heads' slice of every section, in that order)."""
    kd, vd = cfg.gdn_num_qk_heads * cfg.gdn_head_dim, cfg.gdn_num_v_heads * cfg.gdn_head_dim
    return [kd, kd, vd, vd, cfg.gdn_num_v_heads, cfg.gdn_num_v_heads], [kd, kd, vd]


def _qkv_rows(cfg, n: int):
    d = cfg.head_dim
    q = cfg.num_heads * d * (2 if cfg.attention_output_gate else 1) // n
    kv = cfg.num_kv_heads * d // n
    return q, kv


def hf_state_dict(model) -> dict[str, Tensor]:
    """Full (TP-gathered) HF-named state dict of ``model`` on its device (collective under TP)."""
    cfg, g = model.config, model.tp_group
    n = tp_size(g)
    out: dict[str, Tensor] = {"model.embed_tokens.weight": _gather(model.embed_tokens.weight.data, 0, g),
                              "model.norm.weight": model.norm.weight.data}
    if model.lm_head is not None:
        out["lm_head.weight"] = _gather(model.lm_head.data, 0, g)
    for i, layer in enumerate(model.layers):
        p = f"model.layers.{i}."
        out[p + "input_layernorm.weight"] = layer.input_layernorm.weight.data
        out[p + "post_attention_layernorm.weight"] = layer.post_attention_layernorm.weight.data
        mix = layer.self_attention
        if getattr(mix, "tpr_state_kind", "") == "kv":
            qr, kvr = _qkv_rows(cfg, n)
            q, k, v = mix.qkv.weight.data.split((qr, kvr, kvr), 0)
            out[p + "self_attn.q_proj.weight"] = _gather(q, 0, g)
            out[p + "self_attn.k_proj.weight"] = _gather(k, 0, g)
            out[p + "self_attn.v_proj.weight"] = _gather(v, 0, g)
            out[p + "self_attn.o_proj.weight"] = _gather(mix.o_proj.weight.data, 1, g)
            if mix.q_norm is not None:
                out[p + "self_attn.q_norm.weight"] = mix.q_norm.weight.data
                out[p + "self_attn.k_norm.weight"] = mix.k_norm.weight.data
        else:
            proj_s, conv_s = _gdn_sections(cfg, n)
            out[p + "linear_attn.in_proj.weight"] = _gather_sections(mix.in_proj.weight.data,
                                                                     [x // n for x in proj_s], g)
            out[p + "linear_attn.conv1d.weight"] = _gather_sections(mix.conv_weight.data, [x // n for x in conv_s],
                                                                    g).unsqueeze(1)
            out[p + "linear_attn.A_log"] = _gather(mix.A_log.data, 0, g)
            out[p + "linear_attn.dt_bias"] = _gather(mix.dt_bias.data, 0, g)
            out[p + "linear_attn.norm.weight"] = mix.norm_weight.data
            out[p + "linear_attn.out_proj.weight"] = _gather(mix.out_proj.weight.data, 1, g)
        mlp = layer.mlp
        if hasattr(mlp, "fc1"):
            gate, up = mlp.fc1.weight.data.chunk(2, 0)
            out[p + "mlp.gate_proj.weight"] = _gather(gate, 0, g)
            out[p + "mlp.up_proj.weight"] = _gather(up, 0, g)
            out[p + "mlp.down_proj.weight"] = _gather(mlp.fc2.weight.data, 1, g)
        else:
            out.update(_moe_export(mlp, p))
    return {k: v.detach() for k, v in out.items()}


def _moe_export(mlp, p: str) -> dict[str, Tensor]:
    out = {p + "mlp.gate.weight": mlp.router.data}
    ep = 1 if mlp.ep_group is None else dist.get_world_size(mlp.ep_group)
    w1, w2 = mlp.w1.data, mlp.w2.data
    if ep > 1:
        w1 = torch.cat([t for t in _all_gather_list(w1, mlp.ep_group)])
        w2 = torch.cat([t for t in _all_gather_list(w2, mlp.ep_group)])
    for e in range(w1.shape[0]):
        gate, up = w1[e].chunk(2, 0)
        out[p + f"mlp.experts.{e}.gate_proj.weight"] = gate
        out[p + f"mlp.experts.{e}.up_proj.weight"] = up
        out[p + f"mlp.experts.{e}.down_proj.weight"] = w2[e]
    if mlp.shared:
        gate, up = mlp.shared_w1.data.chunk(2, 0)
        out[p + "mlp.shared_expert.gate_proj.weight"] = gate
        out[p + "mlp.shared_expert.up_proj.weight"] = up
        out[p + "mlp.shared_expert.down_proj.weight"] = mlp.shared_w2.data
        out[p + "mlp.shared_expert_gate.weight"] = mlp.shared_gate.data
    return out


def _all_gather_list(t: Tensor, group) -> list[Tensor]:
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, t.contiguous(), group=group)
    return parts


@torch.no_grad()
def load_hf_state_dict(model, sd: dict[str, Tensor], *, strict: bool = True) -> list[str]:
    """Copy an HF-named (unsharded) state dict into ``model``'s TP/EP shards. Returns unused keys."""
    cfg, g = model.config, model.tp_group
    n = tp_size(g)
    used: set[str] = set()

    def take(name: str) -> Tensor:
        if name not in sd:
            raise KeyError(f"checkpoint is missing {name}")
        used.add(name)
        return sd[name]

    def put(param, value: Tensor) -> None:
        if tuple(param.shape) != tuple(value.shape):
            raise ValueError(f"shape mismatch: parameter {tuple(param.shape)} vs checkpoint {tuple(value.shape)}")
        param.data.copy_(value.to(param.dtype))

    put(model.embed_tokens.weight, _split(take("model.embed_tokens.weight"), 0, g))
    put(model.norm.weight, take("model.norm.weight"))
    if model.lm_head is not None:
        put(model.lm_head, _split(take("lm_head.weight"), 0, g))
    for i, layer in enumerate(model.layers):
        p = f"model.layers.{i}."
        put(layer.input_layernorm.weight, take(p + "input_layernorm.weight"))
        put(layer.post_attention_layernorm.weight, take(p + "post_attention_layernorm.weight"))
        mix = layer.self_attention
        if getattr(mix, "tpr_state_kind", "") == "kv":
            q = _split(take(p + "self_attn.q_proj.weight"), 0, g)
            k = _split(take(p + "self_attn.k_proj.weight"), 0, g)
            v = _split(take(p + "self_attn.v_proj.weight"), 0, g)
            put(mix.qkv.weight, torch.cat([q, k, v], 0))
            put(mix.o_proj.weight, _split(take(p + "self_attn.o_proj.weight"), 1, g))
            if mix.q_norm is not None:
                put(mix.q_norm.weight, take(p + "self_attn.q_norm.weight"))
                put(mix.k_norm.weight, take(p + "self_attn.k_norm.weight"))
        else:
            proj_s, conv_s = _gdn_sections(cfg, tp_size(g))
            put(mix.in_proj.weight, _split_sections(take(p + "linear_attn.in_proj.weight"), proj_s, g))
            put(mix.conv_weight, _split_sections(take(p + "linear_attn.conv1d.weight").squeeze(1), conv_s, g))
            put(mix.A_log, _split(take(p + "linear_attn.A_log"), 0, g))
            put(mix.dt_bias, _split(take(p + "linear_attn.dt_bias"), 0, g))
            put(mix.norm_weight, take(p + "linear_attn.norm.weight"))
            put(mix.out_proj.weight, _split(take(p + "linear_attn.out_proj.weight"), 1, g))
        mlp = layer.mlp
        if hasattr(mlp, "fc1"):
            gate = _split(take(p + "mlp.gate_proj.weight"), 0, g)
            up = _split(take(p + "mlp.up_proj.weight"), 0, g)
            put(mlp.fc1.weight, torch.cat([gate, up], 0))
            put(mlp.fc2.weight, _split(take(p + "mlp.down_proj.weight"), 1, g))
        else:
            put(mlp.router, take(p + "mlp.gate.weight"))
            e0 = mlp.ep_rank * mlp.local_experts
            for e in range(mlp.local_experts):
                gate = take(p + f"mlp.experts.{e0 + e}.gate_proj.weight")
                up = take(p + f"mlp.experts.{e0 + e}.up_proj.weight")
                mlp.w1.data[e].copy_(torch.cat([gate, up], 0))
                mlp.w2.data[e].copy_(take(p + f"mlp.experts.{e0 + e}.down_proj.weight"))
            if mlp.shared:
                gate = take(p + "mlp.shared_expert.gate_proj.weight")
                up = take(p + "mlp.shared_expert.up_proj.weight")
                put(mlp.shared_w1, torch.cat([gate, up], 0))
                put(mlp.shared_w2, take(p + "mlp.shared_expert.down_proj.weight"))
                put(mlp.shared_gate, take(p + "mlp.shared_expert_gate.weight"))
    unused = sorted(set(sd) - used)
    if strict and mlp is not None and unused:
        ep_keys = [k for k in unused if ".mlp.experts." in k]
        if len(ep_keys) != len(unused):
            raise KeyError(f"unexpected checkpoint keys: {[k for k in unused if k not in ep_keys][:5]}")
    return unused


def save_safetensors_file(path: str, tensors: dict[str, Tensor], metadata: dict | None = None) -> None:
    from safetensors.torch import save_file

    save_file({k: v.detach().cpu().contiguous() for k, v in tensors.items()}, path, metadata=metadata or {})


def load_safetensors_file(path: str, device="cpu") -> dict[str, Tensor]:
    from safetensors.torch import load_file

    return load_file(path, device=str(device))


def save_checkpoint(directory: str, engine, *, step: int = 0) -> None:
    """HF-format weights (rank 0 of each TP group of DP rank 0) + per-rank optimizer state + meta."""
    os.makedirs(directory, exist_ok=True)
    model = engine.model
    sd = hf_state_dict(model)
    rank = dist.get_rank() if dist.is_initialized() else 0
    if rank == 0:
        save_safetensors_file(os.path.join(directory, "model.safetensors"), sd, {"format": "pt"})
        with open(os.path.join(directory, "meta.json"), "w") as f:
            json.dump({"step": step, "model": model.config.name, "world_size":
                       dist.get_world_size() if dist.is_initialized() else 1}, f)
    torch.save(engine.optimizer.state_dict(), os.path.join(directory, f"optim_rank{rank}.pt"))
    if dist.is_initialized():
        dist.barrier()


def load_checkpoint(directory: str, engine, *, load_optimizer: bool = True) -> int:
    """Load weights (resharded to this engine's TP/EP layout) and, if present, this rank's optimizer state."""
    model = engine.model
    sd = load_safetensors_file(os.path.join(directory, "model.safetensors"))
    load_hf_state_dict(model, sd)
    opt = os.path.join(directory, f"optim_rank{dist.get_rank() if dist.is_initialized() else 0}.pt")
    if load_optimizer and os.path.exists(opt):
        engine.optimizer.load_state_dict(torch.load(opt, map_location=model.norm.weight.device))
    else:
        for a in engine.optimizer.arenas:
            a.master.copy_(a.data.float())
    with open(os.path.join(directory, "meta.json")) as f:
        return int(json.load(f).get("step", 0))
