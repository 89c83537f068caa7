"""Helpers shared by the GPU parity tests: device tensors and oracle configs."""

from __future__ import annotations

import numpy as np

from deciax_b200.config import HeadConfig, KernelFlags, TextConfig
from oracle import clef_oracle as O


def dev(x: np.ndarray, dtype: str):
    """numpy float32 -> CUDA tensor of the compute dtype (bf16 rounds RNE)."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    return t.to(torch.bfloat16) if dtype == "bf16" else t


def host(t) -> np.ndarray:
    import torch

    torch.cuda.synchronize()
    return t.float().cpu().numpy()


def rounded(x: np.ndarray, dtype: str) -> np.ndarray:
    return O.cast(x, dtype)


def oracle_config(c: TextConfig, flags: KernelFlags = KernelFlags()) -> O.TextConfig:
    window = max(flags.layer_window) if flags.layer_window else 0
    return O.TextConfig(
        hidden_size=c.hidden_size,
        intermediate_size=c.intermediate_size,
        num_attention_heads=c.num_attention_heads,
        num_key_value_heads=c.num_key_value_heads,
        head_dim=c.head_dim,
        layer_types=c.layer_types,
        rms_norm_eps=c.rms_norm_eps,
        rope_theta=c.rope_theta,
        partial_rotary_factor=c.partial_rotary_factor,
        linear_num_key_heads=c.linear_num_key_heads,
        linear_num_value_heads=c.linear_num_value_heads,
        linear_key_head_dim=c.linear_key_head_dim,
        linear_value_head_dim=c.linear_value_head_dim,
        linear_conv_kernel_dim=c.linear_conv_kernel_dim,
        attention=O.AttentionFlags(softcap=flags.attn_softcap, window=window),
    )


def oracle_head(h: HeadConfig) -> O.HeadConfig:
    return O.HeadConfig(heads=h.heads, routing_layers=h.routing_layers, layers=h.layers)


def round_tree(tree, dtype: str):
    if isinstance(tree, dict):
        return {k: O.cast(np.asarray(v, np.float32), dtype) for k, v in tree.items()}
    return [round_tree(t, dtype) for t in tree]


def probs_close(actual_logits, expected_logits, arrays, atol: float = 1e-2) -> tuple[float, int]:
    """Max abs option-probability error, and the number of fields whose argmax
    differs while the expected top-2 gap is at least 1e-3."""
    from deciax_b200.synthetic import field_probabilities

    pa = field_probabilities(actual_logits, arrays)
    pe = field_probabilities(expected_logits, arrays)
    err, flips = 0.0, 0
    for fa, fe in zip(pa, pe):
        for a, e in zip(fa, fe):
            err = max(err, float(np.abs(a - e).max()))
            if a.argmax() != e.argmax():
                top = np.sort(e)[::-1]
                if len(top) < 2 or top[0] - top[1] >= 1e-3:
                    flips += 1
    return err, flips
