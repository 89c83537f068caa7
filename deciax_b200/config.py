"""Model configuration: the reference ``TextConfig`` plus the joint-head config.

Same fields, defaults and validation as ``src/deciax/models/qwen3_5/config.py``
(lines 10-75), and the ``joint_head_config.json`` keys read by
``models/clef/model.py:80-83``.  The beyond-reference attention options are
kept apart in :class:`KernelFlags` and default to off.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Literal

LayerType = Literal["linear_attention", "full_attention"]


@dataclass(frozen=True)
class TextConfig:
    hidden_size: int
    intermediate_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    layer_types: tuple[LayerType, ...]
    rms_norm_eps: float
    rope_theta: float
    partial_rotary_factor: float
    vocab_size: int = 0

    def __post_init__(self) -> None:
        sizes = (
            self.hidden_size,
            self.intermediate_size,
            self.num_attention_heads,
            self.num_key_value_heads,
            self.head_dim,
            self.linear_num_key_heads,
            self.linear_num_value_heads,
            self.linear_key_head_dim,
            self.linear_value_head_dim,
            self.linear_conv_kernel_dim,
        )
        if any(size <= 0 for size in sizes):
            raise ValueError("Qwen3.5 dimensions must be positive")
        if self.num_attention_heads % self.num_key_value_heads or self.linear_num_value_heads % self.linear_num_key_heads:
            raise ValueError("Qwen3.5 query/value heads must divide into key head groups")
        if not self.layer_types or set(self.layer_types) - {"linear_attention", "full_attention"}:
            raise ValueError("unsupported Qwen3.5 layer types")
        rotary = int(self.head_dim * self.partial_rotary_factor)
        if rotary <= 0 or rotary % 2 or rotary > self.head_dim:
            raise ValueError("invalid partial rotary dimension")

    @classmethod
    def from_dict(cls, raw: dict[str, Any]) -> "TextConfig":
        c = raw.get("text_config", raw)
        if c.get("attention_bias", False) or c.get("hidden_act", "silu") != "silu" or not c.get("attn_output_gate", True):
            raise ValueError("unsupported Qwen3.5 projection/activation configuration")
        if c.get("num_experts", 0):
            raise ValueError("only dense Qwen3.5 models are supported")
        if len(c["layer_types"]) != c["num_hidden_layers"]:
            raise ValueError("layer_types does not match num_hidden_layers")
        rope = c["rope_parameters"]
        if rope.get("rope_type", "default") != "default":
            raise ValueError("only default RoPE is supported")
        keys = [
            "hidden_size",
            "intermediate_size",
            "num_attention_heads",
            "num_key_value_heads",
            "head_dim",
            "linear_num_key_heads",
            "linear_num_value_heads",
            "linear_key_head_dim",
            "linear_value_head_dim",
            "linear_conv_kernel_dim",
            "rms_norm_eps",
        ]
        return cls(
            **{k: c[k] for k in keys},
            layer_types=tuple(c["layer_types"]),
            rope_theta=rope["rope_theta"],
            partial_rotary_factor=rope.get("partial_rotary_factor", c.get("partial_rotary_factor", 0.25)),
            vocab_size=int(c.get("vocab_size", 0)),
        )

    @classmethod
    def full_attention(cls, *, hidden_size: int, intermediate_size: int, num_attention_heads: int, num_key_value_heads: int,
                       head_dim: int, num_layers: int, vocab_size: int, rms_norm_eps: float = 1e-6,
                       rope_theta: float = 10000.0, partial_rotary_factor: float = 0.25) -> "TextConfig":
        """A config whose layers are all ``full_attention`` (GDN dims unused)."""
        return cls(
            hidden_size=hidden_size,
            intermediate_size=intermediate_size,
            num_attention_heads=num_attention_heads,
            num_key_value_heads=num_key_value_heads,
            head_dim=head_dim,
            linear_num_key_heads=1,
            linear_num_value_heads=1,
            linear_key_head_dim=1,
            linear_value_head_dim=1,
            linear_conv_kernel_dim=1,
            layer_types=("full_attention",) * num_layers,
            rms_norm_eps=rms_norm_eps,
            rope_theta=rope_theta,
            partial_rotary_factor=partial_rotary_factor,
            vocab_size=vocab_size,
        )


@dataclass(frozen=True)
class HeadConfig:
    """``joint_head_config.json``: heads / routing_layers / layers, plus the
    widths the head tensors imply (memory_projection rows, feedforward rows)."""

    heads: int
    routing_layers: int
    layers: int
    width: int
    ffn: int


@dataclass(frozen=True)
class KernelFlags:
    """Beyond-reference options (not in deciax).  Defaults reproduce the reference.

    attn_softcap   softcap * tanh(score / softcap) on scaled attention scores
    layer_window   per-layer causal window (0 = global attention)
    embed_scale    multiply embeddings by this factor in the activation dtype
    """

    attn_softcap: float = 0.0
    layer_window: tuple[int, ...] = field(default_factory=tuple)
    embed_scale: float = 0.0
