"""End-to-end parity of ``ClefCudaModel`` (the C-ABI forward) against the oracle
and against the reference's own golden data.

Bars:
* fp32: final hidden states within 1e-4 relative (rtol 1e-4, atol 1e-4 x the
  largest magnitude) and logits within 1e-4;
* bf16: option probabilities within 1e-2 absolute, argmax identical unless the
  oracle's top-2 gap is below 1e-3;
* the CUDA joint head against Cloudflare's torch head (``clef_head.npz``) and
  the CUDA backbone against Transformers ``Qwen3_5TextModel``.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
from conftest import GOLDEN
from gpu_helpers import oracle_config, oracle_head, probs_close, round_tree

from deciax_b200.config import HeadConfig, KernelFlags, TextConfig
from deciax_b200.model import ClefCudaModel
from deciax_b200.synthetic import BatchSpec, synthetic_batch, synthetic_weights
from oracle import clef_oracle as O

pytestmark = pytest.mark.gpu

SMALL = TextConfig.full_attention(
    hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=64, num_layers=2,
    vocab_size=512,
)
SMALL_HEAD = HeadConfig(heads=4, routing_layers=2, layers=2, width=64, ffn=128)
# head_dim 256 like clef-flash: exercises the d=256 flash-attention kernel
WIDE = TextConfig.full_attention(
    hidden_size=512, intermediate_size=1024, num_attention_heads=2, num_key_value_heads=1, head_dim=256, num_layers=2,
    vocab_size=300, partial_rotary_factor=1.0,
)

# clef-flash's head_dim 256 with the reference default partial rotary 0.25 (fused QKV epilogue)
FLASH = TextConfig.full_attention(
    hidden_size=512, intermediate_size=1024, num_attention_heads=4, num_key_value_heads=2, head_dim=256, num_layers=2,
    vocab_size=300, partial_rotary_factor=0.25,
)

# head_dim 128 with partial rotary 0.25 (rot 32, the 27B-shaped config): the fused QKV epilogue's
# in-chunk rotate-half path
D128 = TextConfig.full_attention(
    hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=128, num_layers=2,
    vocab_size=300, partial_rotary_factor=0.25,
)

SPECS = {
    "ragged": BatchSpec(states=3, seq=256, questions=2, options_per_question=3, lengths=(256, 130, 40), row_bucket=4),
    "full": BatchSpec(states=2, seq=128, questions=4, options_per_question=4),
}


def build(config, head, dtype, seed=1, flags=KernelFlags(), std=0.02, embed_std=1.0):
    top, layers, hp = synthetic_weights(config, head, seed, std=std, embed_std=embed_std)
    top, layers, hp = round_tree(top, dtype), round_tree(layers, dtype), round_tree(hp, dtype)
    model = ClefCudaModel.from_arrays(config, head, top, layers, hp, dtype=dtype, max_seq_len=512, flags=flags)
    return model, (top, layers, hp)


def oracle_forward(weights, arrays, config, head, dtype, flags=KernelFlags()):
    top, layers, hp = weights
    return O.forward(top, layers, hp, arrays, oracle_config(config, flags), oracle_head(head), dtype,
                     embed_scale=flags.embed_scale, return_hidden=True)


@pytest.mark.parametrize("config", [SMALL, WIDE, FLASH, D128], ids=["d64", "d256", "d256-prf025", "d128-prf025"])
@pytest.mark.parametrize("spec", list(SPECS), ids=list(SPECS))
def test_forward_fp32_matches_oracle(config, spec):
    model, weights = build(config, SMALL_HEAD, "fp32")
    arrays = synthetic_batch(SPECS[spec], config.vocab_size, seed=7)
    logits, hidden = model.forward_with_hidden(arrays)
    exp_logits, exp_hidden = oracle_forward(weights, arrays, config, SMALL_HEAD, "fp32")
    valid = arrays["mask"]
    scale = np.abs(exp_hidden[valid]).max()
    np.testing.assert_allclose(hidden[valid], exp_hidden[valid], rtol=1e-4, atol=1e-4 * scale)
    m = arrays["option_mask"]
    np.testing.assert_allclose(logits[m], exp_logits[m], rtol=1e-4, atol=1e-4)
    assert (logits[~m] == -1e9).all()


@pytest.mark.parametrize("config", [SMALL, WIDE, FLASH, D128], ids=["d64", "d256", "d256-prf025", "d128-prf025"])
@pytest.mark.parametrize("spec", list(SPECS), ids=list(SPECS))
def test_forward_bf16_probabilities(config, spec):
    model, weights = build(config, SMALL_HEAD, "bf16")
    arrays = synthetic_batch(SPECS[spec], config.vocab_size, seed=8)
    logits = model.forward(arrays)
    exp_logits, _ = oracle_forward(weights, arrays, config, SMALL_HEAD, "bf16")
    err, flips = probs_close(logits, exp_logits, arrays)
    assert err < 1e-2, err
    assert flips == 0


def test_forward_is_deterministic_and_repeatable():
    model, _ = build(SMALL, SMALL_HEAD, "bf16")
    arrays = synthetic_batch(SPECS["ragged"], SMALL.vocab_size, seed=9)
    a = model.forward(arrays)
    b = model.forward(arrays)
    np.testing.assert_array_equal(a, b)


def test_padding_does_not_leak():
    """Padded tokens and padded batch rows cannot change real rows' logits."""
    model, _ = build(SMALL, SMALL_HEAD, "fp32")
    arrays = synthetic_batch(SPECS["ragged"], SMALL.vocab_size, seed=10)
    base = model.forward(arrays)
    changed = {k: v.copy() for k, v in arrays.items()}
    changed["input_ids"][~changed["mask"]] = 17
    again = model.forward(changed)
    np.testing.assert_allclose(again[:3], base[:3], rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("config,dtype", [(SMALL, "fp32"), (SMALL, "bf16"), (WIDE, "bf16")])
def test_poisoned_scratch_changes_nothing(config, dtype):
    """Sanitizer substitute: with every scratch buffer filled with NaN bytes
    before the forward (CLEF_DEBUG_POISON), logits and real hidden states stay
    bit-identical, so no kernel reads memory it has not written first (tile
    padding, stale rows of an earlier larger batch, unwritten head buffers)."""
    model, _ = build(config, SMALL_HEAD, dtype)
    big = synthetic_batch(SPECS["ragged"], config.vocab_size, seed=13)
    small = synthetic_batch(SPECS["full"], config.vocab_size, seed=14)
    model.forward(big)  # the workspace is sized for the larger batch first
    for arrays in (small, big):
        base_logits, base_hidden = model.forward_with_hidden(arrays)
        model.set_debug(poison=True)
        logits, hidden = model.forward_with_hidden(arrays)
        model.set_debug(poison=False)
        np.testing.assert_array_equal(logits, base_logits)
        valid = arrays["mask"]
        np.testing.assert_array_equal(hidden[valid], base_hidden[valid])
        assert np.isfinite(logits[arrays["option_mask"]]).all()


def test_beyond_reference_flags_match_oracle():
    flags = KernelFlags(attn_softcap=20.0, layer_window=(64, 0), embed_scale=2.0)
    model, weights = build(SMALL, SMALL_HEAD, "fp32", flags=flags)
    arrays = synthetic_batch(SPECS["ragged"], SMALL.vocab_size, seed=11)
    logits, hidden = model.forward_with_hidden(arrays)
    # The oracle applies the per-layer window through a single flag: compare a
    # config whose every layer is windowed.
    flags_all = KernelFlags(attn_softcap=20.0, layer_window=(64, 64), embed_scale=2.0)
    model2, _ = build(SMALL, SMALL_HEAD, "fp32", flags=flags_all)
    logits2, hidden2 = model2.forward_with_hidden(arrays)
    exp_logits, exp_hidden = oracle_forward(weights, arrays, SMALL, SMALL_HEAD, "fp32", flags_all)
    valid = arrays["mask"]
    scale = np.abs(exp_hidden[valid]).max()
    np.testing.assert_allclose(hidden2[valid], exp_hidden[valid], rtol=1e-4, atol=1e-4 * scale)
    assert np.abs(hidden[valid] - hidden2[valid]).max() > 0  # layer 1 global vs windowed differs


def test_bad_token_id_is_value_error():
    model, _ = build(SMALL, SMALL_HEAD, "bf16")
    arrays = synthetic_batch(SPECS["full"], SMALL.vocab_size, seed=12)
    arrays["input_ids"][0, 0] = SMALL.vocab_size
    with pytest.raises(ValueError):
        model.forward(arrays)


def test_joint_head_matches_cloudflare_fixture():
    """tests/clef/test_head.py:11-29 of the reference, through the CUDA head (fp32)."""
    f = np.load(GOLDEN / "clef_head.npz")
    p = {k[6:]: f[k] for k in f.files if k.startswith("param.")}
    a = {k[6:]: f[k] for k in f.files if k.startswith("array.")}
    emb = f["embedding"]
    config = TextConfig.full_attention(hidden_size=32, intermediate_size=64, num_attention_heads=2, num_key_value_heads=1,
                                       head_dim=16, num_layers=1, vocab_size=emb.shape[0])
    head = HeadConfig(heads=4, routing_layers=2, layers=2, width=16, ffn=32)
    top, layers, _ = synthetic_weights(config, head, 0)
    top = {"embedding": emb, "lm_head": emb, "norm": top["norm"]}
    model = ClefCudaModel.from_arrays(config, head, top, layers, p, dtype="fp32", max_seq_len=128)
    out = model.forward_head(a, f["hidden"])
    for i in range(3):
        expected = f[f"expected.{i}"]
        np.testing.assert_allclose(out[i, : len(expected)], expected, atol=3e-6, rtol=3e-5)
    changed = np.where(a["mask"][..., None], f["hidden"], 10000.0)
    second = model.forward_head(a, changed)
    np.testing.assert_allclose(out[:3], second[:3], atol=1e-6)


def test_backbone_matches_transformers_fixture():
    """tests/test_qwen3_5.py:43-87 of the reference (all-full-attention variant), through CUDA fp32."""
    f = np.load(GOLDEN / "qwen35_backbone_full.npz")
    raw = json.loads(bytes(f["config_json"]).decode())
    config = TextConfig.from_dict(raw)
    config = TextConfig(**{**config.__dict__, "vocab_size": raw["vocab_size"]})
    params = {k[6:]: f[k] for k in f.files if k.startswith("param.")}
    head = HeadConfig(heads=2, routing_layers=1, layers=1, width=16, ffn=32)
    _, _, hp = synthetic_weights(config, head, 0)
    top = {"embedding": params["embed_tokens.weight"], "lm_head": params["embed_tokens.weight"], "norm": params["norm.weight"]}
    layers = []
    for i in range(len(config.layer_types)):
        pre = f"layers.{i}."
        layers.append(O.layer_weights({k[len(pre):]: v for k, v in params.items() if k.startswith(pre)}, O.TextConfig(
            hidden_size=32, intermediate_size=64, num_attention_heads=4, num_key_value_heads=2, head_dim=16)))
    model = ClefCudaModel.from_arrays(config, head, top, layers, hp, dtype="fp32", max_seq_len=256)
    ids, mask = f["ids"], f["mask"]
    b, s = ids.shape
    arrays = {
        "input_ids": ids, "mask": mask, "lexical_ids": np.zeros((b, 128), np.int32),
        "lexical_spans": np.tile(np.array([[[0, 1]]], np.int32), (b, 1, 1)),
        "question_spans": np.tile(np.array([[[0, 2]]], np.int32), (b, 1, 1)), "question_mask": np.ones((b, 1), bool),
        "types": np.ones((b, 1), np.int32), "option_spans": np.tile(np.array([[[2, 3]]], np.int32), (b, 1, 1)),
        "option_mask": np.ones((b, 1), bool), "option_field": np.zeros((b, 1), np.int32),
    }
    _, hidden = model.forward_with_hidden(arrays)
    valid = mask.astype(bool)
    np.testing.assert_allclose(hidden[valid], f["expected"][valid], atol=3e-6, rtol=3e-5)
