"""Gated DeltaNet (linear_attention layers) on the GPU against the oracle.

* ``clef_op_gdn_core`` (conv + SiLU, L2 norms, gates, chunked delta rule,
  gated RMSNorm x SiLU(z)) against ``delta_net_core`` of the oracle
  (models/qwen3_5/text.py:48-67, kernels/gdn/reference.py:40-92) at every
  supported head dim, key/value head ratios 1-4, lengths around the 64-token
  chunk (1, 63, 64, 65, 70, 100, 130) and up to 2048, and conv widths 1-6
  (BF16 at head dim 128 runs the tensor-core conv, prep and chain passes,
  every other case the CUDA-core kernel);
* whole models with GDN layers: the Transformers ``Qwen3_5TextModel`` fixture
  of the reference test (tests/test_qwen3_5.py:43-87: 3 GDN + 1 full layer)
  through the CUDA FP32 path, and synthetic mixed stacks against the oracle in
  FP32 and BF16.

Bars: FP32 within 1e-4 relative (atol 1e-4 x the largest magnitude); BF16
core outputs within 2e-2 relative + 1e-2 x the largest magnitude (the output
passes four bf16 roundings, each may differ by one step); BF16 model option
probabilities within 1e-2.
"""

from __future__ import annotations

import ctypes
import json

import numpy as np
import pytest
from conftest import GOLDEN
from gpu_helpers import dev, host, oracle_config, oracle_head, probs_close, round_tree

from deciax_b200 import _lib
from deciax_b200.config import HeadConfig, TextConfig
from deciax_b200.model import ClefCudaModel
from deciax_b200.synthetic import BatchSpec, synthetic_batch, synthetic_weights
from oracle import clef_oracle as O

pytestmark = pytest.mark.gpu


def core_case(b, s, nh, nv, dh, width, dtype, seed):
    rng = np.random.default_rng(seed)
    nk, nvd = nh * dh, nv * dh
    n = 2 * nk + 2 * nvd + 2 * nv
    proj = O.cast(rng.standard_normal((b, s, n)).astype(np.float32), dtype)
    conv = O.cast((rng.standard_normal((2 * nk + nvd, width)) * 0.5).astype(np.float32), dtype)
    A_log = O.cast(np.log(rng.uniform(0.01, 0.3, nv)).astype(np.float32), dtype)
    dt_bias = O.cast(rng.normal(0, 0.5, nv).astype(np.float32), dtype)
    norm_w = O.cast((1 + rng.normal(0, 0.1, dh)).astype(np.float32), dtype)
    cols = np.cumsum([0, nk, nk, nvd, nvd, nv, nv])
    names = ("q", "k", "v", "in_proj_z", "in_proj_a", "in_proj_b")
    projs = {k: proj[..., cols[i]:cols[i + 1]] for i, k in enumerate(names)}
    p = {"q.conv": conv[:nk], "k.conv": conv[nk:2 * nk], "v.conv": conv[2 * nk:], "A_log": A_log, "dt_bias": dt_bias,
         "norm.weight": norm_w}
    c = O.TextConfig(hidden_size=8, intermediate_size=8, num_attention_heads=1, num_key_value_heads=1, head_dim=8,
                     linear_num_key_heads=nh, linear_num_value_heads=nv, linear_key_head_dim=dh, linear_value_head_dim=dh,
                     linear_conv_kernel_dim=width)
    expected = O.delta_net_core(p, projs, c, dtype)
    return proj, conv, A_log, dt_bias, norm_w, expected


CASES = [  # b, s, nh, nv, dh, width
    (2, 130, 2, 6, 8, 4),
    (1, 1, 1, 1, 16, 4),
    (2, 63, 1, 2, 32, 3),
    (1, 64, 2, 2, 64, 4),
    (2, 65, 1, 3, 64, 1),
    (1, 130, 2, 4, 128, 4),
    (3, 200, 1, 2, 128, 4),
    (1, 2048, 1, 2, 128, 4),  # 32 chunks of state recurrence (BF16: the tensor-core passes)
    # BF16 tensor-core passes: one value head per key head, four per key head, a lone token,
    # an exact chunk, and a conv wider than four taps
    (2, 1, 2, 2, 128, 4),
    (2, 64, 2, 2, 128, 3),
    (1, 100, 1, 4, 128, 2),
    (1, 70, 1, 1, 128, 6),
]


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
@pytest.mark.parametrize("case", CASES, ids=[f"b{c[0]}s{c[1]}h{c[2]}v{c[3]}d{c[4]}w{c[5]}" for c in CASES])
def test_gdn_core_matches_oracle(case, dtype):
    b, s, nh, nv, dh, width = case
    proj, conv, A_log, dt_bias, norm_w, expected = core_case(b, s, nh, nv, dh, width, dtype, seed=sum(case))
    lib = _lib.load()
    import torch

    ldp = -(-proj.shape[-1] // 16) * 16  # 16-byte rows in either dtype
    padded = np.zeros((b * s, ldp), np.float32)
    padded[:, : proj.shape[-1]] = proj.reshape(b * s, -1)
    tp, tc, ta, tb, tw = (dev(x, dtype) for x in (padded, conv, A_log, dt_bias, norm_w))
    out = torch.full((b * s, nv * dh), float("nan"), device="cuda", dtype=tp.dtype)
    dt = _lib.DTYPE_BF16 if dtype == "bf16" else _lib.DTYPE_F32
    _lib.check(lib.clef_op_gdn_core(dt, tp.data_ptr(), ldp, tc.data_ptr(), width, ta.data_ptr(), tb.data_ptr(),
                                    tw.data_ptr(), out.data_ptr(), b, s, nh, nv, dh, ctypes.c_float(1e-6), None))
    got = host(out).reshape(expected.shape)
    scale = float(np.abs(expected).max())
    if dtype == "fp32":
        np.testing.assert_allclose(got, expected, rtol=1e-4, atol=1e-4 * scale)
    else:
        np.testing.assert_allclose(got, expected, rtol=2e-2, atol=1e-2 * scale)
        assert np.abs(got - expected).mean() < 2e-3 * scale


def test_gdn_core_aligned_keys_with_weak_decay_are_stable():
    """tests/test_qwen3_5.py:90-102 of the reference through the CUDA core: every
    token's q = k (constant projections through a unit width-1 conv), decay
    g = -exp(A_log) softplus(a + dt_bias) ~ -1e-5 and beta = sigmoid(b) ~ 0.996,
    130 tokens, head dim 128, BF16.  The chunk's triangular system is then
    nearly singular; the output must stay finite and match the oracle."""
    lib = _lib.load()
    import torch

    b, s, nh, nv, dh, width, dtype = 1, 130, 2, 2, 128, 1, "bf16"
    nk, nvd = nh * dh, nv * dh
    n = 2 * nk + 2 * nvd + 2 * nv
    proj = np.ones((b, s, n), np.float32)
    # v differs across channels (the same for every token), so the gated norm
    # at the end does not flatten the recurrence's output into a constant
    proj[..., 2 * nk: 2 * nk + nvd] = np.random.default_rng(9).standard_normal(nvd).astype(np.float32)
    proj[..., 2 * nk + 2 * nvd: 2 * nk + 2 * nvd + nv] = np.log(np.e - 1)  # a: softplus(a + 0) = 1
    proj[..., 2 * nk + 2 * nvd + nv:] = np.log(0.996 / 0.004)  # b: beta ~ 0.996
    proj = O.cast(proj, dtype)
    conv = O.cast(np.ones((2 * nk + nvd, width), np.float32), dtype)
    A_log = O.cast(np.full(nv, np.log(1e-5), np.float32), dtype)
    dt_bias = O.cast(np.zeros(nv, np.float32), dtype)
    norm_w = O.cast(np.ones(dh, np.float32), dtype)
    cols = np.cumsum([0, nk, nk, nvd, nvd, nv, nv])
    names = ("q", "k", "v", "in_proj_z", "in_proj_a", "in_proj_b")
    projs = {k: proj[..., cols[i]:cols[i + 1]] for i, k in enumerate(names)}
    p = {"q.conv": conv[:nk], "k.conv": conv[nk:2 * nk], "v.conv": conv[2 * nk:], "A_log": A_log, "dt_bias": dt_bias,
         "norm.weight": norm_w}
    c = O.TextConfig(hidden_size=8, intermediate_size=8, num_attention_heads=1, num_key_value_heads=1, head_dim=8,
                     linear_num_key_heads=nh, linear_num_value_heads=nv, linear_key_head_dim=dh, linear_value_head_dim=dh,
                     linear_conv_kernel_dim=width)
    expected = O.delta_net_core(p, projs, c, dtype)
    ldp = -(-n // 16) * 16
    padded = np.zeros((b * s, ldp), np.float32)
    padded[:, :n] = proj.reshape(b * s, -1)
    tp, tc, ta, tb, tw = (dev(x, dtype) for x in (padded, conv, A_log, dt_bias, norm_w))
    out = torch.full((b * s, nv * dh), float("nan"), device="cuda", dtype=tp.dtype)
    _lib.check(lib.clef_op_gdn_core(_lib.DTYPE_BF16, tp.data_ptr(), ldp, tc.data_ptr(), width, ta.data_ptr(),
                                    tb.data_ptr(), tw.data_ptr(), out.data_ptr(), b, s, nh, nv, dh, ctypes.c_float(1e-6), None))
    got = host(out).reshape(expected.shape)
    assert np.isfinite(got).all() and np.isfinite(expected).all()
    scale = float(np.abs(expected).max())
    np.testing.assert_allclose(got, expected, rtol=2e-2, atol=1e-2 * scale)


def test_gdn_core_rejects_unsupported_head_dim():
    lib = _lib.load()
    import torch

    x = torch.zeros(1024, device="cuda")
    status = lib.clef_op_gdn_core(_lib.DTYPE_F32, x.data_ptr(), 1024, x.data_ptr(), 4, x.data_ptr(), x.data_ptr(),
                                  x.data_ptr(), x.data_ptr(), 1, 4, 1, 1, 24, ctypes.c_float(1e-6), None)
    assert status == _lib.CLEF_EINVAL


def test_mixed_backbone_matches_transformers_fixture():
    """tests/test_qwen3_5.py:43-87 of the reference (3 GDN + 1 full layer), CUDA FP32."""
    f = np.load(GOLDEN / "qwen35_backbone_mixed.npz")
    raw = json.loads(bytes(f["config_json"]).decode())
    config = TextConfig.from_dict(raw)
    config = TextConfig(**{**config.__dict__, "vocab_size": raw["vocab_size"]})
    params = {k[6:]: f[k] for k in f.files if k.startswith("param.")}
    head = HeadConfig(heads=2, routing_layers=1, layers=1, width=16, ffn=32)
    _, _, hp = synthetic_weights(TextConfig.full_attention(hidden_size=32, intermediate_size=64, num_attention_heads=2,
                                                           num_key_value_heads=1, head_dim=8, num_layers=1, vocab_size=8),
                                 head, 0)
    top = {"embedding": params["embed_tokens.weight"], "lm_head": params["embed_tokens.weight"], "norm": params["norm.weight"]}
    model = ClefCudaModel(config, head, dtype="fp32", max_seq_len=256)
    for k in ("embedding", "lm_head", "norm"):
        model.upload(k, top[k])
    for key, value in params.items():
        if key.startswith("layers."):
            _, i, rest = key.split(".", 2)
            # checkpoint names, fused in_proj_qkv / conv1d split inside the library
            model.upload(f"layers.{i}.{rest.replace('linear_attn.', 'mixer.').replace('self_attn.', 'mixer.')}", value)
    for k, v in hp.items():
        model.upload("head." + k, v)
    model.finalize()
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


MIXED = TextConfig(
    hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
    linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=128, linear_value_head_dim=128,
    linear_conv_kernel_dim=4, layer_types=("linear_attention", "full_attention", "linear_attention"),
    rms_norm_eps=1e-6, rope_theta=10000.0, partial_rotary_factor=0.25, vocab_size=512,
)
HEAD = HeadConfig(heads=4, routing_layers=2, layers=2, width=64, ffn=128)
SPEC = BatchSpec(states=3, seq=256, questions=2, options_per_question=3, lengths=(256, 130, 40), row_bucket=4)


def build(dtype, seed=4):
    top, layers, hp = (round_tree(t, dtype) for t in synthetic_weights(MIXED, HEAD, seed, embed_std=1.0))
    model = ClefCudaModel.from_arrays(MIXED, HEAD, top, layers, hp, dtype=dtype, max_seq_len=512)
    return model, (top, layers, hp)


def test_mixed_model_fp32_matches_oracle():
    model, (top, layers, hp) = build("fp32")
    arrays = synthetic_batch(SPEC, MIXED.vocab_size, seed=5)
    logits, hidden = model.forward_with_hidden(arrays)
    exp_logits, exp_hidden = O.forward(top, layers, hp, arrays, oracle_config(MIXED), oracle_head(HEAD), "fp32",
                                       return_hidden=True)
    valid = arrays["mask"]
    scale = np.abs(exp_hidden[valid]).max()
    np.testing.assert_allclose(hidden[valid], exp_hidden[valid], rtol=1e-4, atol=1e-4 * scale)
    m = arrays["option_mask"]
    np.testing.assert_allclose(logits[m], exp_logits[m], rtol=1e-4, atol=1e-4)


def test_mixed_model_bf16_probabilities():
    model, (top, layers, hp) = build("bf16")
    arrays = synthetic_batch(SPEC, MIXED.vocab_size, seed=6)
    logits = model.forward(arrays)
    exp_logits, _ = O.forward(top, layers, hp, arrays, oracle_config(MIXED), oracle_head(HEAD), "bf16", return_hidden=True)
    err, flips = probs_close(logits, exp_logits, arrays)
    assert err < 1e-2 and flips == 0, (err, flips)


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_mixed_model_poisoned_scratch_changes_nothing(dtype):
    """Gated DeltaNet layers under CLEF_DEBUG_POISON: NaN-filled scratch
    buffers (the packed projection's padding columns included) change no bit
    of the logits or real hidden states."""
    model, _ = build(dtype)
    arrays = synthetic_batch(SPEC, MIXED.vocab_size, seed=8)
    base_logits, base_hidden = model.forward_with_hidden(arrays)
    model.set_debug(poison=True)
    logits, hidden = model.forward_with_hidden(arrays)
    np.testing.assert_array_equal(logits, base_logits)
    valid = arrays["mask"]
    np.testing.assert_array_equal(hidden[valid], base_hidden[valid])


def test_mixed_model_padding_does_not_leak():
    model, _ = build("fp32")
    arrays = synthetic_batch(SPEC, MIXED.vocab_size, seed=7)
    base = model.forward(arrays)
    changed = {k: v.copy() for k, v in arrays.items()}
    changed["input_ids"][~changed["mask"]] = 11
    np.testing.assert_allclose(model.forward(changed)[:3], base[:3], rtol=1e-6, atol=1e-6)
