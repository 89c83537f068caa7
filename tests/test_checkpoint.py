"""Host-side checkpoint validation (``read_checkpoint``), on CPU: the plan of
what ``from_pretrained`` uploads and the reference's rejections
(models/clef/model.py:51-57, weights.py:26-101, qwen3_5/config.py:51-75)."""

from __future__ import annotations

import json

import numpy as np
import pytest
from checkpoint_helpers import mixed_config, write_checkpoint, write_safetensors

from deciax_b200.model import read_checkpoint, safetensors_header, safetensors_tensors
from deciax_b200.synthetic import synthetic_weights


@pytest.fixture
def weights():
    config, head = mixed_config()
    top, layers, hp = synthetic_weights(config, head, seed=3, dtype="bf16")
    return config, head, top, layers, hp


def test_plan_maps_hub_keys_to_library_names(tmp_path, weights):
    config, head, top, layers, hp = weights
    extra = {"model.visual.blocks.0.attn.qkv.weight": np.zeros((4, 4), np.float32)}
    d = write_checkpoint(tmp_path / "ckpt", config, head, top, layers, hp, shards=3, extra=extra)
    plan = read_checkpoint(d)
    assert plan.config == config and plan.head_config == head and plan.pad_token_id == 1
    names = {k: v for m in plan.backbone.values() for k, v in m.items()}
    assert len(plan.backbone) == 3
    assert names["model.language_model.embed_tokens.weight"] == "embedding"
    assert names["lm_head.weight"] == "lm_head"
    assert names["model.language_model.norm.weight"] == "norm"
    # the fused Gated DeltaNet tensors keep their names; the library splits them
    assert names["model.language_model.layers.0.linear_attn.in_proj_qkv.weight"] == "layers.0.mixer.in_proj_qkv.weight"
    assert names["model.language_model.layers.0.linear_attn.conv1d.weight"] == "layers.0.mixer.conv1d.weight"
    assert names["model.language_model.layers.0.linear_attn.A_log"] == "layers.0.mixer.A_log"
    assert names["model.language_model.layers.1.self_attn.q_proj.weight"] == "layers.1.mixer.q_proj.weight"
    assert names["model.language_model.layers.1.mlp.down_proj.weight"] == "layers.1.mlp.down_proj.weight"
    assert "model.visual.blocks.0.attn.qkv.weight" not in names  # the vision tower is skipped (weights.py:84-85)


def test_safetensors_round_trip(tmp_path):
    import ml_dtypes

    a = (np.arange(12, dtype=np.float32) / 7).reshape(3, 4)
    t = {"x": a.astype(ml_dtypes.bfloat16), "y": a, "z": a.astype(np.float16)}
    write_safetensors(tmp_path / "t.safetensors", t)
    got = dict(safetensors_tensors(tmp_path / "t.safetensors"))
    np.testing.assert_array_equal(np.asarray(got["x"], np.float32), a.astype(ml_dtypes.bfloat16).astype(np.float32))
    np.testing.assert_array_equal(got["y"], a)
    np.testing.assert_array_equal(got["z"], a.astype(np.float16).astype(np.float32))


def test_unexpected_backbone_key_is_rejected(tmp_path, weights):
    config, head, top, layers, hp = weights
    d = write_checkpoint(tmp_path / "c", config, head, top, layers, hp, extra={"model.mtp.weight": np.zeros(2, np.float32)})
    with pytest.raises(ValueError, match="unexpected backbone tensor: model.mtp.weight"):
        read_checkpoint(d)
    d = write_checkpoint(tmp_path / "c2", config, head, top, layers, hp,
                         extra={"model.language_model.layers.7.mlp.up_proj.weight": np.zeros(2, np.float32)})
    with pytest.raises(ValueError, match="unexpected backbone tensor"):
        read_checkpoint(d)


@pytest.mark.parametrize("drop", [("model.language_model.norm.weight",), ("lm_head.weight",)])
def test_missing_top_tensor_is_incomplete(tmp_path, weights, drop):
    config, head, top, layers, hp = weights
    d = write_checkpoint(tmp_path / "c", config, head, top, layers, hp, drop=drop)
    with pytest.raises(ValueError, match="incomplete Clef text checkpoint"):
        read_checkpoint(d)


def test_layer_without_tensors_is_incomplete(tmp_path, weights):
    config, head, top, layers, hp = weights
    keys = [k for k in __import__("checkpoint_helpers").checkpoint_tensors(config, top, layers)
            if k.startswith("model.language_model.layers.1.")]
    d = write_checkpoint(tmp_path / "c", config, head, top, layers, hp, drop=tuple(keys))
    with pytest.raises(ValueError, match="incomplete Clef text checkpoint"):
        read_checkpoint(d)


def test_missing_pad_token(tmp_path, weights):
    config, head, top, layers, hp = weights
    d = write_checkpoint(tmp_path / "c", config, head, top, layers, hp, pad_token=False)
    with pytest.raises(ValueError, match="missing pad token"):
        read_checkpoint(d)


@pytest.mark.parametrize("change,message", [
    ({"attention_bias": True}, "unsupported Qwen3.5 projection/activation configuration"),
    ({"num_experts": 8}, "only dense Qwen3.5 models are supported"),
    ({"num_hidden_layers": 3}, "layer_types does not match num_hidden_layers"),
    ({"rope_parameters": {"rope_type": "yarn", "rope_theta": 1e4}}, "only default RoPE is supported"),
    ({"layer_types": ["linear_attention", "sliding_attention"]}, "unsupported Qwen3.5 layer types"),
])
def test_config_rejections(tmp_path, weights, change, message):
    config, head, top, layers, hp = weights
    d = write_checkpoint(tmp_path / "c", config, head, top, layers, hp)
    raw = json.loads((d / "config.json").read_text())
    raw["text_config"].update(change)
    (d / "config.json").write_text(json.dumps(raw))
    with pytest.raises(ValueError, match=message):
        read_checkpoint(d)


def test_corrupt_safetensors_offsets(tmp_path, weights):
    config, head, top, layers, hp = weights
    d = write_checkpoint(tmp_path / "c", config, head, top, layers, hp, shards=1)
    f = d / "model-00001-of-00001.safetensors"
    f.write_bytes(f.read_bytes()[:-16])  # truncated data section
    with pytest.raises(ValueError, match="invalid data offsets"):
        safetensors_header(f)
    with pytest.raises(ValueError, match="invalid data offsets"):
        read_checkpoint(d)
