"""Write small synthetic Clef checkpoint directories in the Hub layout that
``ClefCudaModel.from_pretrained`` reads (models/clef/model.py:51-85,
weights.py:70-101): ``config.json`` with ``text_config`` and
``rope_parameters``, ``tokenizer.json``, backbone safetensors shards with
``model.safetensors.index.json``, ``joint_head_config.json`` and
``joint_head.safetensors``.  Gated DeltaNet layers are written with the
checkpoint's fused ``linear_attn.in_proj_qkv`` and ``linear_attn.conv1d``
tensors; attention layers under ``self_attn``.
"""

from __future__ import annotations

import json
import struct
from pathlib import Path

import ml_dtypes
import numpy as np

from deciax_b200.config import HeadConfig, TextConfig


def write_safetensors(path: Path, tensors: dict[str, np.ndarray]) -> None:
    """8-byte little-endian header length, JSON header, raw little-endian data."""
    header, blobs, offset = {}, [], 0
    for key, a in tensors.items():
        a = np.ascontiguousarray(a)
        dtype = {np.dtype(ml_dtypes.bfloat16): "BF16", np.dtype(np.float32): "F32", np.dtype(np.float16): "F16"}[a.dtype]
        blob = a.tobytes()
        header[key] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [offset, offset + len(blob)]}
        blobs.append(blob)
        offset += len(blob)
    text = json.dumps(header).encode()
    text += b" " * (-len(text) % 8)
    path.write_bytes(struct.pack("<Q", len(text)) + text + b"".join(blobs))


def config_json(config: TextConfig) -> dict:
    c = config
    return {"architectures": ["Qwen3_5ForConditionalGeneration"], "text_config": {
        "hidden_size": c.hidden_size, "intermediate_size": c.intermediate_size,
        "num_attention_heads": c.num_attention_heads, "num_key_value_heads": c.num_key_value_heads, "head_dim": c.head_dim,
        "linear_num_key_heads": c.linear_num_key_heads, "linear_num_value_heads": c.linear_num_value_heads,
        "linear_key_head_dim": c.linear_key_head_dim, "linear_value_head_dim": c.linear_value_head_dim,
        "linear_conv_kernel_dim": c.linear_conv_kernel_dim, "rms_norm_eps": c.rms_norm_eps,
        "num_hidden_layers": len(c.layer_types), "layer_types": list(c.layer_types), "vocab_size": c.vocab_size,
        "hidden_act": "silu", "attention_bias": False, "attn_output_gate": True,
        "rope_parameters": {"rope_type": "default", "rope_theta": c.rope_theta,
                            "partial_rotary_factor": c.partial_rotary_factor}}}


def write_tokenizer(path: Path, vocab: int, pad: bool = True) -> None:
    from tokenizers import Tokenizer, models, pre_tokenizers

    words = {"[UNK]": 0}
    if pad:
        words["<|endoftext|>"] = 1
    for i in range(len(words), vocab):
        words[f"w{i}"] = i
    tok = Tokenizer(models.WordLevel(vocab=words, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.save(str(path))


def checkpoint_tensors(config: TextConfig, top: dict, layers: list[dict]) -> dict[str, np.ndarray]:
    """Hub key -> array for the split weights of ``synthetic_weights``: the
    inverse of the renames and the q/k/v split of weights.py:43-57."""
    out = {
        "model.language_model.embed_tokens.weight": top["embedding"],
        "lm_head.weight": top["lm_head"],
        "model.language_model.norm.weight": top["norm"],
    }
    for i, (kind, p) in enumerate(zip(config.layer_types, layers, strict=True)):
        pre = f"model.language_model.layers.{i}."
        mixer = "linear_attn." if kind == "linear_attention" else "self_attn."
        for name, value in p.items():
            if name.startswith("mixer.") and kind == "linear_attention" and name[6:] in (
                    "q.weight", "k.weight", "v.weight", "q.conv", "k.conv", "v.conv"):
                continue
            out[pre + name.replace("mixer.", mixer)] = value
        if kind == "linear_attention":
            out[pre + "linear_attn.in_proj_qkv.weight"] = np.concatenate(
                [p["mixer.q.weight"], p["mixer.k.weight"], p["mixer.v.weight"]])
            out[pre + "linear_attn.conv1d.weight"] = np.concatenate(
                [p["mixer.q.conv"], p["mixer.k.conv"], p["mixer.v.conv"]])[:, None, :]
    return out


def write_checkpoint(directory: Path, config: TextConfig, head: HeadConfig, top: dict, layers: list[dict],
                     head_weights: dict, *, shards: int = 2, extra: dict | None = None, drop: tuple[str, ...] = (),
                     pad_token: bool = True) -> Path:
    """A checkpoint directory holding these weights, the backbone split over
    ``shards`` files.  ``extra`` adds keys (e.g. a vision-tower tensor the
    loader must skip); ``drop`` removes Hub keys."""
    directory.mkdir(parents=True, exist_ok=True)
    (directory / "config.json").write_text(json.dumps(config_json(config)))
    write_tokenizer(directory / "tokenizer.json", config.vocab_size, pad=pad_token)
    tensors = checkpoint_tensors(config, top, layers) | (extra or {})
    for key in drop:
        tensors.pop(key)
    keys = sorted(tensors)
    weight_map = {}
    for s in range(shards):
        name = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        part = {k: tensors[k] for k in keys[s::shards]}
        write_safetensors(directory / name, part)
        weight_map |= {k: name for k in part}
    (directory / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    (directory / "joint_head_config.json").write_text(
        json.dumps({"heads": head.heads, "routing_layers": head.routing_layers, "layers": head.layers}))
    write_safetensors(directory / "joint_head.safetensors", head_weights)
    return directory


def mixed_config() -> tuple[TextConfig, HeadConfig]:
    """One Gated DeltaNet layer and one full-attention layer (the reference
    test's hybrid stack, shortened)."""
    config = TextConfig(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                        linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=32,
                        linear_value_head_dim=32, linear_conv_kernel_dim=4,
                        layer_types=("linear_attention", "full_attention"), rms_norm_eps=1e-6, rope_theta=10000.0,
                        partial_rotary_factor=0.25, vocab_size=300)
    return config, HeadConfig(heads=4, routing_layers=1, layers=1, width=64, ffn=128)
