"""Model configurations of the Qwen3.5 hybrid family (gated DeltaNet + gated full attention).

``qwen35_27b`` is the shape the benchmarks use: 64 layers, hidden 5120, every 4th
layer full attention (24 Q / 4 KV heads, head_dim 256, partial RoPE over 64 dims,
theta 1e7, sigmoid output gate), the others gated DeltaNet (16 K / 48 V heads of
dim 128, conv kernel 4), SwiGLU MLP 17408, vocab 248320, one MTP layer.
"""
from __future__ import annotations

from dataclasses import dataclass, field, asdict


@dataclass
class HybridConfig:
    vocab_size: int = 248320
    hidden_size: int = 5120
    intermediate_size: int = 17408
    num_layers: int = 64
    full_attention_interval: int = 4
    num_attention_heads: int = 24
    num_key_value_heads: int = 4
    head_dim: int = 256
    partial_rotary_factor: float = 0.25
    rope_theta: float = 1.0e7
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 48
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    rms_norm_eps: float = 1e-6
    num_mtp_layers: int = 1
    max_position: int = 262144
    rope_scaling: dict | None = None  # e.g. {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": ...}
    name: str = "qwen35-27b"
    layer_types: list = field(default_factory=list)

    def __post_init__(self):
        if not self.layer_types:
            self.layer_types = [
                "full_attention" if (i + 1) % self.full_attention_interval == 0 else "linear_attention"
                for i in range(self.num_layers)
            ]

    @property
    def rot_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def full_layer_ids(self) -> list[int]:
        return [i for i, t in enumerate(self.layer_types) if t == "full_attention"]

    def to_dict(self) -> dict:
        return asdict(self)


def qwen35_27b(**overrides) -> HybridConfig:
    return HybridConfig(**overrides)


def tiny(num_layers: int = 4, **overrides) -> HybridConfig:
    """Small config with the kernel-supported head geometry (head_dim 256, dk = dv = 128)."""
    base = dict(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_layers=num_layers,
                num_attention_heads=6, num_key_value_heads=1, head_dim=256, linear_num_key_heads=2,
                linear_num_value_heads=6, max_position=8192, name="qwen35-tiny")
    base.update(overrides)
    return HybridConfig(**base)


CONFIGS = {"qwen35-27b": qwen35_27b, "qwen35-tiny": tiny}
