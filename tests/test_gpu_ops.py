"""Kernel-level parity: each CUDA kernel through the C ABI vs the CPU oracle.

Tolerances: bf16 outputs within 2^-7 relative (one bf16 rounding step;
the GPU and the oracle sum fp32 products in different orders), fp32 outputs
within 1e-4 relative.  Shapes include M/N/K tails, ragged masks and padding.
"""

from __future__ import annotations

import numpy as np
import pytest
from gpu_helpers import dev, host

from deciax_b200 import _lib
from oracle import clef_oracle as O

pytestmark = pytest.mark.gpu
F32 = np.float32
BF16_RTOL = 2.0**-7


def lib():
    return _lib.load()


def dt_code(dtype: str) -> int:
    return _lib.DTYPE_BF16 if dtype == "bf16" else _lib.DTYPE_F32


def ptr(t) -> int:
    return t.data_ptr() if t is not None else None


def run_gemm(dtype, epi, a, b, out, ldo, bias=None, res=None, ldr=0):
    m, k = a.shape
    n = b.shape[0]
    st = lib().clef_op_gemm(dt_code(dtype), epi, m, n, k, ptr(a), ptr(b), ptr(out), ldo, ptr(bias), ptr(res), ldr, None)
    _lib.check(st)


GEMM_SHAPES = [(128, 256, 64), (256, 512, 256), (300, 200, 136), (1000, 768, 512), (2048, 3584, 1024), (64, 96, 32)]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
@pytest.mark.parametrize("epi", ["store", "bias", "residual", "f32"])
def test_gemm_bf16_tcgen05(m, n, k, epi):
    import torch

    rng = np.random.default_rng(m * 7 + n * 3 + k)
    a = O.bf16(rng.standard_normal((m, k)).astype(F32))
    b = O.bf16(rng.standard_normal((n, k)).astype(F32) * F32(0.05))
    acc = (a.astype(np.float64) @ b.astype(np.float64).T).astype(F32)
    A, B = dev(a, "bf16"), dev(b, "bf16")
    if epi == "f32":
        out = torch.zeros((m, n), dtype=torch.float32, device="cuda")
        run_gemm("bf16", 3, A, B, out, n)
        np.testing.assert_allclose(host(out), acc, rtol=1e-4, atol=1e-4 * np.abs(acc).max())
        return
    out = torch.zeros((m, n), dtype=torch.bfloat16, device="cuda")
    if epi == "residual":
        r = O.bf16(rng.standard_normal((m, n)).astype(F32))
        out.copy_(dev(r, "bf16"))
        run_gemm("bf16", 2, A, B, out, n, res=out, ldr=n)  # in place, as the layer does
        expected = O.bf16(r + O.bf16(acc))
        # Two roundings: T(acc) may round the other way when the fp32 sums differ
        # in their last bits (one step of acc), and T(r + T(acc)) then rounds
        # again (one step of the sum): two bf16 steps of the larger magnitude.
        scale = 2 * (np.abs(r) + np.abs(acc))
    else:
        bias = O.bf16(rng.standard_normal(n).astype(F32)) if epi == "bias" else None
        run_gemm("bf16", 0, A, B, out, n, bias=dev(bias, "bf16") if bias is not None else None)
        expected = O.bf16(acc + (bias if bias is not None else 0))
        scale = np.abs(expected)
    got = host(out)
    # One bf16 step of the output scale, plus a floor for the fp32 accumulation
    # order (K products of magnitude ~0.05 summed in a different order).
    tol = BF16_RTOL * scale + 1e-3
    bad = np.abs(got - expected) > tol
    if bad.any():
        i = np.unravel_index(np.argmax(np.abs(got - expected) - tol), got.shape)
        raise AssertionError(f"{bad.sum()} elements out of tolerance; worst at {i}: got {got[i]}, expected {expected[i]}, "
                             f"fp32 acc {acc[i]}")
    assert np.mean(got != expected) < 0.02  # almost every element bit-identical


@pytest.mark.parametrize("n", [128, 768])
def test_gemm_bf16_rows_do_not_depend_on_the_launch(n):
    """A row's result is bit-identical whether it runs among 1000 rows (CTA
    pairs for N >= 256), 300 rows or 64 rows (one CTA): the K order of the
    tcgen05 accumulation does not depend on M, so batching cannot change an
    answer."""
    import torch

    rng = np.random.default_rng(n)
    k = 512
    a = O.bf16(rng.standard_normal((1000, k)).astype(F32))
    b = O.bf16(rng.standard_normal((n, k)).astype(F32) * F32(0.05))
    A, B = dev(a, "bf16"), dev(b, "bf16")
    full = torch.zeros((1000, n), dtype=torch.bfloat16, device="cuda")
    run_gemm("bf16", 0, A, B, full, n)
    for rows in (300, 64, 1):
        part = torch.zeros((rows, n), dtype=torch.bfloat16, device="cuda")
        sub = A[100 : 100 + rows].contiguous()
        run_gemm("bf16", 0, sub, B, part, n)
        assert torch.equal(part, full[100 : 100 + rows]), rows


@pytest.mark.parametrize("m,f,k", [(128, 128, 64), (300, 256, 136), (1024, 1792, 512)])
def test_gemm_bf16_swiglu_epilogue(m, f, k):
    import torch

    rng = np.random.default_rng(f + k)
    x = O.bf16(rng.standard_normal((m, k)).astype(F32))
    gate = O.bf16(rng.standard_normal((f, k)).astype(F32) * F32(0.1))
    up = O.bf16(rng.standard_normal((f, k)).astype(F32) * F32(0.1))
    packed = np.zeros((2 * f, k), F32)
    for j0 in range(0, f, 128):
        packed[2 * j0 : 2 * j0 + 128] = gate[j0 : j0 + 128]
        packed[2 * j0 + 128 : 2 * j0 + 256] = up[j0 : j0 + 128]
    out = torch.zeros((m, f), dtype=torch.bfloat16, device="cuda")
    run_gemm("bf16", 1, dev(x, "bf16"), dev(packed, "bf16"), out, f)
    g = O.bf16(x.astype(np.float64) @ gate.T.astype(np.float64))
    u = O.bf16(x.astype(np.float64) @ up.T.astype(np.float64))
    expected = O.bf16(O.bf16(O.silu(g)) * u)
    np.testing.assert_allclose(host(out), expected, rtol=2 * BF16_RTOL, atol=2e-3)


@pytest.mark.parametrize("d,prf,hq,hkv", [(256, 0.25, 2, 1), (128, 0.5, 4, 2), (64, 1.0, 4, 2), (256, 1.0, 1, 1),
                                          (128, 0.25, 4, 2), (64, 0.5, 2, 2)])
def test_gemm_qkv_fused_epilogue(d, prf, hq, hkv):
    """QKV GEMM + q/k RMSNorm + partial RoPE + sigmoid(gate) in the epilogue vs the oracle."""
    import torch

    rng = np.random.default_rng(d + hq)
    b, s, k = 2, 128, 256
    n = hq * 2 * d + 2 * hkv * d
    x = O.bf16(rng.standard_normal((b * s, k)).astype(F32))
    w = O.bf16(rng.standard_normal((n, k)).astype(F32) * F32(0.1))
    qw = O.bf16(rng.standard_normal(d).astype(F32) * F32(0.1))
    kw = O.bf16(rng.standard_normal(d).astype(F32) * F32(0.1))
    X, Wt, QW, KW = dev(x, "bf16"), dev(w, "bf16"), dev(qw, "bf16"), dev(kw, "bf16")
    out = torch.zeros((b * s, n), dtype=torch.bfloat16, device="cuda")
    st = lib().clef_op_gemm_qkv(ptr(X), ptr(Wt), ptr(out), b * s, k, hq, hkv, d, prf, 10000.0, s, ptr(QW), ptr(KW), 1e-6, None)
    _lib.check(st)
    got = host(out).reshape(b, s, n)
    proj = O.bf16(x.astype(np.float64) @ w.T.astype(np.float64)).reshape(b, s, n)
    raw = proj[..., : hq * 2 * d].reshape(b, s, hq, 2 * d)
    q, gate = raw[..., :d], raw[..., d:]
    kk = proj[..., hq * 2 * d : hq * 2 * d + hkv * d].reshape(b, s, hkv, d)
    v = proj[..., hq * 2 * d + hkv * d :]
    q, kk = O.rms(q, qw, 1e-6, "bf16"), O.rms(kk, kw, 1e-6, "bf16")
    rot = int(d * prf)
    inv = O.rope_inv_freq(rot, 10000.0)
    q = np.concatenate((O.apply_rope(q[..., :rot], inv, "bf16"), q[..., rot:]), -1)
    kk = np.concatenate((O.apply_rope(kk[..., :rot], inv, "bf16"), kk[..., rot:]), -1)
    got_raw = got[..., : hq * 2 * d].reshape(b, s, hq, 2 * d)
    tol = dict(rtol=2 * BF16_RTOL, atol=1e-2)
    np.testing.assert_allclose(got_raw[..., :d], q, **tol)
    np.testing.assert_allclose(got_raw[..., d:], O.bf16(O.sigmoid(gate)), **tol)
    np.testing.assert_allclose(got[..., hq * 2 * d : hq * 2 * d + hkv * d].reshape(b, s, hkv, d), kk, **tol)
    np.testing.assert_allclose(got[..., hq * 2 * d + hkv * d :], v, rtol=BF16_RTOL, atol=1e-3)


@pytest.mark.parametrize("epi", ["store", "residual", "f32"])
def test_gemm_f32_simt(epi):
    import torch

    rng = np.random.default_rng(5)
    m, n, k = 300, 200, 136
    a = rng.standard_normal((m, k)).astype(F32)
    b = rng.standard_normal((n, k)).astype(F32) * F32(0.05)
    acc = (a.astype(np.float64) @ b.astype(np.float64).T).astype(F32)
    out = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    if epi == "residual":
        r = rng.standard_normal((m, n)).astype(F32)
        out.copy_(dev(r, "fp32"))
        run_gemm("fp32", 2, dev(a, "fp32"), dev(b, "fp32"), out, n, res=out, ldr=n)
        expected = r + acc
    else:
        run_gemm("fp32", 0 if epi == "store" else 3, dev(a, "fp32"), dev(b, "fp32"), out, n)
        expected = acc
    np.testing.assert_allclose(host(out), expected, rtol=1e-5, atol=1e-5)


def test_gemm_rejects_misaligned_k():
    import torch

    a = torch.zeros((128, 30), dtype=torch.bfloat16, device="cuda")
    b = torch.zeros((128, 30), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((128, 128), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        run_gemm("bf16", 0, a, b, out, 128)


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("rows,dim", [(333, 3584), (17, 40), (1, 256)])
def test_rmsnorm(dtype, rows, dim):
    import torch

    rng = np.random.default_rng(rows + dim)
    x = O.cast(rng.standard_normal((rows, dim)).astype(F32) * F32(3), dtype)
    w = O.cast(rng.standard_normal(dim).astype(F32) * F32(0.1), dtype)
    out = torch.empty((rows, dim), dtype=torch.bfloat16 if dtype == "bf16" else torch.float32, device="cuda")
    X, Wt = dev(x, dtype), dev(w, dtype)  # keep alive: the caching allocator would otherwise alias them
    _lib.check(lib().clef_op_rmsnorm(dt_code(dtype), ptr(X), ptr(Wt), ptr(out), rows, dim, 1e-6, None))
    expected = O.rms(x, w, 1e-6, dtype)
    if dtype == "bf16":
        np.testing.assert_allclose(host(out), expected, rtol=BF16_RTOL, atol=1e-6)
    else:
        np.testing.assert_allclose(host(out), expected, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
@pytest.mark.parametrize("d,prf", [(64, 0.25), (256, 0.25), (128, 1.0), (16, 0.5)])
def test_qk_norm_rope(dtype, d, prf):
    rng = np.random.default_rng(d)
    b, s, hq, hkv = 2, 70, 4, 2
    n = hq * 2 * d + 2 * hkv * d
    qkv = O.cast(rng.standard_normal((b, s, n)).astype(F32), dtype)
    qw = O.cast(rng.standard_normal(d).astype(F32) * F32(0.1), dtype)
    kw = O.cast(rng.standard_normal(d).astype(F32) * F32(0.1), dtype)
    t = dev(qkv.reshape(b * s, n), dtype)
    QW, KW = dev(qw, dtype), dev(kw, dtype)  # keep alive: the caching allocator would otherwise alias them
    st = lib().clef_op_qk_norm_rope(dt_code(dtype), ptr(t), b, s, hq, hkv, d, prf, 10000.0, ptr(QW), ptr(KW), 1e-6, None)
    _lib.check(st)
    got = host(t).reshape(b, s, n)
    raw = qkv[..., : hq * 2 * d].reshape(b, s, hq, 2 * d)
    q, k = raw[..., :d], qkv[..., hq * 2 * d : hq * 2 * d + hkv * d].reshape(b, s, hkv, d)
    q, k = O.rms(q, qw, 1e-6, dtype), O.rms(k, kw, 1e-6, dtype)
    rot = int(d * prf)
    inv = O.rope_inv_freq(rot, 10000.0)
    q = np.concatenate((O.apply_rope(q[..., :rot], inv, dtype), q[..., rot:]), -1)
    k = np.concatenate((O.apply_rope(k[..., :rot], inv, dtype), k[..., rot:]), -1)
    got_q = got[..., : hq * 2 * d].reshape(b, s, hq, 2 * d)
    tol = dict(rtol=2 * BF16_RTOL, atol=1e-2) if dtype == "bf16" else dict(rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got_q[..., :d], q, **tol)
    np.testing.assert_array_equal(got_q[..., d:], raw[..., d:])  # gate untouched
    np.testing.assert_allclose(got[..., hq * 2 * d : hq * 2 * d + hkv * d].reshape(b, s, hkv, d), k, **tol)
    np.testing.assert_array_equal(got[..., hq * 2 * d + hkv * d :], qkv[..., hq * 2 * d + hkv * d :])  # v untouched


def attention_case(dtype, d, s, softcap=0.0, window=0, lengths=None, seed=0, qscale=1.0, hq=4, hkv=2):
    import torch

    rng = np.random.default_rng(seed + d + s)
    b = 2
    n = hq * 2 * d + 2 * hkv * d
    qkv = rng.standard_normal((b, s, n)).astype(F32)
    qkv[..., : hq * 2 * d] *= F32(qscale)  # large scores: the running max moves and O is rescaled
    qkv = O.cast(qkv, dtype)
    lengths = lengths or [s, max(1, s - 37)]
    mask = np.arange(s)[None] < np.array(lengths)[:, None]
    out = torch.zeros((b * s, hq * d), dtype=torch.bfloat16 if dtype == "bf16" else torch.float32, device="cuda")
    m = torch.from_numpy(mask.astype(np.uint8)).cuda()
    QKV = dev(qkv.reshape(b * s, n), dtype)
    st = lib().clef_op_attention(dt_code(dtype), ptr(QKV), ptr(m), ptr(out), b, s, hq, hkv, d, softcap, window, None)
    _lib.check(st)
    raw = qkv[..., : hq * 2 * d].reshape(b, s, hq, 2 * d)
    q, gate = raw[..., :d], raw[..., d:]
    k = qkv[..., hq * 2 * d : hq * 2 * d + hkv * d].reshape(b, s, hkv, d)
    v = qkv[..., hq * 2 * d + hkv * d :].reshape(b, s, hkv, d)
    flags = O.AttentionFlags(softcap=softcap, window=window)
    att = O.attention(q, k, v, mask, causal=True, dtype=dtype, flags=flags)
    expected = O.cast(att * O.cast(O.sigmoid(gate), dtype), dtype).reshape(b, s, hq * d)
    return host(out).reshape(b, s, hq * d), expected


@pytest.mark.parametrize("hq,hkv", [(2, 2), (8, 2)])
def test_attention_bf16_d256_group_sizes(hq, hkv):
    """head_dim 256 with one query head per key/value head and with four."""
    got, expected = attention_case("bf16", 256, 257, hq=hq, hkv=hkv, seed=7)
    np.testing.assert_allclose(got, expected, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("s", [130, 257])
def test_attention_bf16_flash(d, s):
    got, expected = attention_case("bf16", d, s)
    np.testing.assert_allclose(got, expected, rtol=2e-2, atol=2e-2)
    assert np.abs(got - expected).mean() < 2e-3


@pytest.mark.parametrize("d", [128, 256])
def test_attention_bf16_long_rows_with_rescales(d):
    """Many 64-key tiles per query tile, scores large enough that the running
    max moves by more than the lazy-rescale margin (head_dim 128 keeps P in
    tensor memory; 256 in shared memory)."""
    got, expected = attention_case("bf16", d, 1024, lengths=[1024, 700], qscale=6.0, seed=3)
    np.testing.assert_allclose(got, expected, rtol=2e-2, atol=2e-2)
    assert np.abs(got - expected).mean() < 2e-3


@pytest.mark.parametrize("d", [8, 64, 256])
def test_attention_fp32_exact(d):
    got, expected = attention_case("fp32", d, 130)
    np.testing.assert_allclose(got, expected, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("s,lengths", [(384, [384, 300]), (2048, [2048, 1999])])
def test_attention_bf16_d256_long_sequences(s, lengths):
    """head_dim 256 at 384 tokens (three 128-row tiles, each leaving through
    TMA stores) and at the benchmark layer's 2048, with a ragged second row."""
    got, expected = attention_case("bf16", 256, s, lengths=lengths, seed=5)
    np.testing.assert_allclose(got, expected, rtol=2e-2, atol=2e-2)
    assert np.abs(got - expected).mean() < 2e-3


@pytest.mark.parametrize("dtype,d", [("bf16", 64), ("bf16", 128), ("bf16", 256), ("fp32", 64)])
def test_attention_beyond_reference_flags(dtype, d):
    got, expected = attention_case(dtype, d, 200, softcap=5.0, window=48)
    tol = dict(rtol=2e-2, atol=2e-2) if dtype == "bf16" else dict(rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(got, expected, **tol)


@pytest.mark.parametrize("dtype,d", [("bf16", 64), ("bf16", 128), ("bf16", 256), ("fp32", 64)])
def test_attention_length_one_row(dtype, d):
    """A state whose only valid key is key 0: every later query attends to it alone."""
    got, expected = attention_case(dtype, d, 66, lengths=[1, 66])
    tol = dict(rtol=2e-2, atol=2e-2) if dtype == "bf16" else dict(rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(got, expected, **tol)
