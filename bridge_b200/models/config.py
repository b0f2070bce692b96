"""Model configurations: Qwen3 dense, hybrid GDN/attention, hybrid MoE.

Presets cover the shapes the benchmarks name:

* ``tiny``           -- 2 layers, hidden 256, 4q/2kv heads of 64, FFN 512, vocab 1024 (CPU correctness)
* ``qwen3_4b``       -- 36 layers, hidden 2560, 32q/8kv heads of 128, FFN 9728, vocab 151936, tied head
* ``hybrid_gdn_2b``  -- 24 layers of [GDN, GDN, GDN, gated attention], hidden 2048, GDN 16 qk / 32 v heads
                        of 128 with conv 4, attention 16q/2kv of 256, FFN 5632, vocab 151936
* ``qwen3_next_24l`` -- the hybrid layout with 512 experts (FFN 512) top-10 + one shared expert
"""

from __future__ import annotations

from dataclasses import dataclass, field, replace


@dataclass(frozen=True)
class ModelConfig:
    vocab_size: int = 1024
    hidden_size: int = 256
    intermediate_size: int = 512
    num_layers: int = 2
    num_heads: int = 4
    num_kv_heads: int = 2
    head_dim: int = 64
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    qk_norm: bool = True
    tie_word_embeddings: bool = True
    # Layer layout: "attention" or "gdn" per layer (None -> all attention).
    layer_types: tuple[str, ...] | None = None
    attention_output_gate: bool = False
    # Gated DeltaNet
    gdn_num_qk_heads: int = 16
    gdn_num_v_heads: int = 32
    gdn_head_dim: int = 128
    gdn_conv_kernel: int = 4
    gdn_chunk_size: int = 64
    # MoE (num_experts == 0 -> dense SwiGLU MLP)
    num_experts: int = 0
    moe_top_k: int = 0
    moe_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    router_aux_loss_coef: float = 0.0
    init_std: float = 0.02
    name: str = "custom"

    def __post_init__(self) -> None:
        if self.num_heads % self.num_kv_heads:
            raise ValueError("num_heads must be a multiple of num_kv_heads")
        if self.layer_types is not None and len(self.layer_types) != self.num_layers:
            raise ValueError("layer_types must have one entry per layer")
        if self.layer_types is not None and any(t not in ("attention", "gdn") for t in self.layer_types):
            raise ValueError("layer_types entries must be 'attention' or 'gdn'")

    @property
    def types(self) -> tuple[str, ...]:
        return self.layer_types or ("attention",) * self.num_layers

    @property
    def attention_layer_numbers(self) -> tuple[int, ...]:
        return tuple(i + 1 for i, t in enumerate(self.types) if t == "attention")

    @property
    def gdn_layer_numbers(self) -> tuple[int, ...]:
        return tuple(i + 1 for i, t in enumerate(self.types) if t == "gdn")

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def param_count(self) -> int:
        """Approximate total parameter count (unsharded)."""
        h, d = self.hidden_size, self.head_dim
        total = self.vocab_size * h * (1 if self.tie_word_embeddings else 2) + h
        for t in self.types:
            total += 2 * h
            if t == "attention":
                q = self.num_heads * d * (2 if self.attention_output_gate else 1)
                total += h * (q + 2 * self.num_kv_heads * d) + self.num_heads * d * h
                total += 2 * d if self.qk_norm else 0
            else:
                kd, vd = self.gdn_num_qk_heads * self.gdn_head_dim, self.gdn_num_v_heads * self.gdn_head_dim
                total += h * (2 * kd + 2 * vd + 2 * self.gdn_num_v_heads) + vd * h
                total += (2 * kd + vd) * self.gdn_conv_kernel + 2 * self.gdn_num_v_heads + self.gdn_head_dim
            if self.is_moe:
                total += h * self.num_experts + self.num_experts * 3 * h * self.moe_intermediate_size
                total += 3 * h * self.shared_expert_intermediate_size + h
            else:
                total += 3 * h * self.intermediate_size
        return total


def _hybrid_types(n: int) -> tuple[str, ...]:
    return tuple("attention" if (i % 4) == 3 else "gdn" for i in range(n))


PRESETS: dict[str, ModelConfig] = {
    "tiny": ModelConfig(name="tiny"),
    "qwen3_4b": ModelConfig(
        name="qwen3_4b", vocab_size=151936, hidden_size=2560, intermediate_size=9728, num_layers=36,
        num_heads=32, num_kv_heads=8, head_dim=128, rope_theta=1e6, tie_word_embeddings=True,
    ),
    "hybrid_gdn_2b": ModelConfig(
        name="hybrid_gdn_2b", vocab_size=151936, hidden_size=2048, intermediate_size=5632, num_layers=24,
        num_heads=16, num_kv_heads=2, head_dim=256, layer_types=_hybrid_types(24), attention_output_gate=True,
        gdn_num_qk_heads=16, gdn_num_v_heads=32, gdn_head_dim=128, gdn_conv_kernel=4, gdn_chunk_size=64,
        tie_word_embeddings=False,
    ),
    "qwen3_next_24l": ModelConfig(
        name="qwen3_next_24l", vocab_size=151936, hidden_size=2048, intermediate_size=512, num_layers=24,
        num_heads=16, num_kv_heads=2, head_dim=256, layer_types=_hybrid_types(24), attention_output_gate=True,
        gdn_num_qk_heads=16, gdn_num_v_heads=32, gdn_head_dim=128, num_experts=512, moe_top_k=10,
        moe_intermediate_size=512, shared_expert_intermediate_size=512, tie_word_embeddings=False,
    ),
    "tiny_hybrid": ModelConfig(
        name="tiny_hybrid", vocab_size=1024, hidden_size=256, intermediate_size=512, num_layers=4,
        num_heads=4, num_kv_heads=2, head_dim=64, layer_types=_hybrid_types(4), attention_output_gate=True,
        gdn_num_qk_heads=2, gdn_num_v_heads=4, gdn_head_dim=32, gdn_conv_kernel=4, gdn_chunk_size=16,
    ),
    "tiny_moe": ModelConfig(
        name="tiny_moe", vocab_size=1024, hidden_size=256, intermediate_size=128, num_layers=4,
        num_heads=4, num_kv_heads=2, head_dim=64, layer_types=_hybrid_types(4), attention_output_gate=True,
        gdn_num_qk_heads=2, gdn_num_v_heads=4, gdn_head_dim=32, gdn_conv_kernel=4, gdn_chunk_size=16,
        num_experts=8, moe_top_k=2, moe_intermediate_size=128, shared_expert_intermediate_size=128,
    ),
}


def get_config(name: str, **overrides) -> ModelConfig:
    try:
        base = PRESETS[name]
    except KeyError as exc:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}") from exc
    if "num_layers" in overrides and "layer_types" not in overrides and base.layer_types is not None:
        n = overrides["num_layers"]
        if n > len(base.layer_types):
            raise ValueError(f"{name} defines {len(base.layer_types)} layer types; cannot build {n} layers")
        overrides["layer_types"] = base.layer_types[:n]   # a truncated hybrid keeps its layer pattern
    return replace(base, **overrides) if overrides else base
