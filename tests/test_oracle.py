"""Pins for the CPU oracle against the reference's own golden data.

These mirror the reference tests so that the oracle -- the checker every GPU
parity test uses -- is itself anchored:

* ``tests/clef/test_head.py:11-29``: joint head vs Cloudflare's torch head
  (``clef_head.npz``), atol 3e-6 / rtol 3e-5, plus padding invariance;
* ``tests/test_qwen3_5.py:43-87``: backbone vs Transformers ``Qwen3_5TextModel``
  (mixed GDN + full attention), atol 3e-6 / rtol 3e-5;
* ``tests/test_qwen3_5.py:17-24``: chunked GDN vs the token recurrence;
* ``tests/test_qwen3_5.py:27-40``: causal GQA attention vs a dense softmax;
* ``tests/test_qwen3_5.py:90-102``: the aligned-key / weak-decay regression.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
from conftest import GOLDEN

from oracle import clef_oracle as O


def _backbone(name: str):
    f = np.load(GOLDEN / f"{name}.npz")
    c = O.TextConfig.from_dict(json.loads(bytes(f["config_json"]).decode()))
    params = {k[6:]: f[k] for k in f.files if k.startswith("param.")}
    return f, c, params


@pytest.mark.parametrize("name", ["qwen35_backbone_mixed", "qwen35_backbone_full"])
def test_backbone_matches_transformers(name: str) -> None:
    f, c, params = _backbone(name)
    h = f["embedded"]
    for i, kind in enumerate(c.layer_types):
        pre = f"layers.{i}."
        p = O.layer_weights({k[len(pre) :]: v for k, v in params.items() if k.startswith(pre)}, c)
        h = O.layer(p, h, f["mask"], c, linear_attention=kind == "linear_attention", dtype="fp32")
    out = O.rms(h, params["norm.weight"], c.rms_norm_eps, "fp32")
    valid = f["mask"].astype(bool)
    np.testing.assert_allclose(out[valid], f["expected"][valid], atol=3e-6, rtol=3e-5)


def test_embedding_matches_transformers() -> None:
    f, _, params = _backbone("qwen35_backbone_full")
    np.testing.assert_array_equal(O.embed(params["embed_tokens.weight"], f["ids"], "fp32"), f["embedded"])


def _head_fixture():
    f = np.load(GOLDEN / "clef_head.npz")
    p = {k[6:]: f[k] for k in f.files if k.startswith("param.")}
    a = {k[6:]: f[k] for k in f.files if k.startswith("array.")}
    lex = O.means(f["embedding"][a["lexical_ids"]], a["lexical_spans"], "fp32")
    return f, p, a, lex


def test_joint_head_matches_cloudflare_with_mixed_schema_padding() -> None:
    f, p, a, lex = _head_fixture()
    out = O.head_forward(p, f["hidden"], lex, a, heads=4, routing_layers=2, layers=2, dtype="fp32")
    for i in range(3):
        expected = f[f"expected.{i}"]
        np.testing.assert_allclose(out[i, : len(expected)], expected, atol=3e-6, rtol=3e-5)
    changed = np.where(a["mask"][..., None], f["hidden"], 10000.0)
    second = O.head_forward(p, changed, lex, a, heads=4, routing_layers=2, layers=2, dtype="fp32")
    np.testing.assert_allclose(out[:3], second[:3], atol=1e-6)


def test_joint_head_bf16_close_to_fp32() -> None:
    """The bf16 emulation stays near the fp32 result on the fixture (sanity)."""
    f, p, a, lex = _head_fixture()
    full = O.head_forward(p, f["hidden"], lex, a, heads=4, routing_layers=2, layers=2, dtype="fp32")
    pb = {k: O.bf16(v) for k, v in p.items()}
    half = O.head_forward(pb, O.bf16(f["hidden"]), O.bf16(lex), a, heads=4, routing_layers=2, layers=2, dtype="bf16")
    m = a["option_mask"]
    assert np.abs(full[m] - half[m]).max() < 0.1


@pytest.mark.parametrize("length", [1, 63, 64, 65, 130])
def test_chunked_matches_recurrence(length: int) -> None:
    rng = np.random.default_rng(12)
    q, k, v = (rng.normal(size=(2, length, 3, 8)).astype(np.float32) for _ in range(3))
    g = -rng.uniform(0, 3, (2, length, 3)).astype(np.float32)
    beta = rng.uniform(0, 1, (2, length, 3)).astype(np.float32)
    np.testing.assert_allclose(O.gdn_chunked(q, k, v, g, beta, "fp32"), O.gdn_recurrent(q, k, v, g, beta, "fp32"), atol=2e-6, rtol=2e-5)


def test_blocked_attention_matches_dense() -> None:
    rng = np.random.default_rng(3)
    s, d = 139, 8
    q = rng.normal(size=(2, s, 4, d)).astype(np.float32)
    k, v = (rng.normal(size=(2, s, 2, d)).astype(np.float32) for _ in range(2))
    mask = np.arange(s)[None] < np.array([s, 97])[:, None]
    keys, values = (np.repeat(x, 2, axis=2) for x in (k, v))
    logits = np.einsum("bqhd,bkhd->bhqk", q, keys) * d**-0.5
    causal = np.arange(s)[:, None] >= np.arange(s)[None, :]
    logits = np.where(mask[:, None, None, :] & causal, logits, -1e30)
    e = np.exp(logits - logits.max(-1, keepdims=True))
    expected = np.einsum("bhqk,bkhd->bqhd", e / e.sum(-1, keepdims=True), values)
    np.testing.assert_allclose(O.attention(q, k, v, mask, causal=True, dtype="fp32"), expected, atol=1e-6, rtol=1e-5)


def test_aligned_keys_with_weak_decay_are_stable() -> None:
    q = k = O.bf16(np.ones((1, 130, 2, 128), np.float32))
    v = q.copy()
    g = np.full((1, 130, 2), -1e-5, np.float32)
    beta = O.bf16(np.full(g.shape, 0.996, np.float32))
    actual = O.gdn_chunked(q, k, v, g, beta, "bf16")
    expected = O.gdn_recurrent(q, k, v, g, beta, "bf16")
    assert np.isfinite(actual).all()
    np.testing.assert_allclose(actual, expected, atol=1e-3, rtol=1e-3)


def test_beyond_reference_flags_default_off() -> None:
    """Softcap/window flags at their defaults reproduce plain attention; on, they change it."""
    rng = np.random.default_rng(4)
    q = rng.normal(size=(1, 40, 2, 16)).astype(np.float32) * 4
    k, v = (rng.normal(size=(1, 40, 1, 16)).astype(np.float32) * 4 for _ in range(2))
    mask = np.ones((1, 40), bool)
    base = O.attention(q, k, v, mask, causal=True, dtype="fp32")
    np.testing.assert_array_equal(base, O.attention(q, k, v, mask, causal=True, dtype="fp32", flags=O.AttentionFlags()))
    capped = O.attention(q, k, v, mask, causal=True, dtype="fp32", flags=O.AttentionFlags(softcap=5.0))
    windowed = O.attention(q, k, v, mask, causal=True, dtype="fp32", flags=O.AttentionFlags(window=8))
    assert np.abs(capped - base).max() > 1e-3 and np.abs(windowed - base).max() > 1e-3
    np.testing.assert_allclose(windowed[:, :8], base[:, :8], atol=1e-6)
