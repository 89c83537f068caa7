"""The allocation-free q/k-norm + RoPE entry point against the allocating one.

``clef_op_qk_norm_rope_noalloc`` serves callers that cannot allocate device
memory (a framework that owns all device buffers, or a loop that must avoid
cudaMalloc's device synchronisation); it keeps its cos/sin tables in a fixed
array inside the library.  This file is named so pytest collects it last.
Each test runs two calls in a row with different shapes, so a table left
behind by the first call cannot satisfy the second.

Both entry points evaluate cos and sin of the same float32 angles
(float32(pos) * inv_freq) in double precision and round once to float32 --
the allocating one on the host, the allocation-free one on the device -- and
then run the same kernel.  Two double-precision evaluations of one angle can
differ by an ulp or two of a double, which changes the float32 result only
for a value within that distance of a float32 rounding boundary; the tables
of these cases have none (the closest value is 360 double ulps away), so the
outputs must be bit-identical.  The long case (4096 positions, 128 rotary
pairs) makes the angles grow large enough that an off-by-one position or
frequency index would show.
"""

from __future__ import annotations

import numpy as np
import pytest

from deciax_b200 import _lib
from oracle import clef_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(dtype, b, s, hq, hkv, d, seed):
    rng = np.random.default_rng(seed)
    n = hq * 2 * d + 2 * hkv * d
    qkv = O.cast(rng.standard_normal((b * s, n)).astype(np.float32), dtype)
    qw = O.cast(rng.standard_normal(d).astype(np.float32) * np.float32(0.1), dtype)
    kw = O.cast(rng.standard_normal(d).astype(np.float32) * np.float32(0.1), dtype)
    return qkv, qw, kw


def _device(x, dtype):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    return t.to(torch.bfloat16) if dtype == "bf16" else t


def _run(fn, dtype, qkv, b, s, hq, hkv, d, prf, qw, kw):
    code = _lib.DTYPE_BF16 if dtype == "bf16" else _lib.DTYPE_F32
    _lib.check(fn(code, qkv.data_ptr(), b, s, hq, hkv, d, prf, 10000.0, qw.data_ptr(), kw.data_ptr(), 1e-6, None))


def _oracle(qkv, b, s, hq, hkv, d, prf, qw, kw, dtype):
    """q/k RMSNorm(1 + w) and partial rotate-half RoPE (models/qwen3_5/text.py:79-88, nn.py:31-44)."""
    x = qkv.reshape(b, s, -1)
    raw = x[..., : hq * 2 * d].reshape(b, s, hq, 2 * d)
    q, k = raw[..., :d], x[..., hq * 2 * d : hq * 2 * d + hkv * d].reshape(b, s, hkv, d)
    q, k = O.rms(q, qw, 1e-6, dtype), O.rms(k, kw, 1e-6, dtype)
    rot = int(d * prf)
    inv = O.rope_inv_freq(rot, 10000.0)
    q = np.concatenate((O.apply_rope(q[..., :rot], inv, dtype), q[..., rot:]), -1)
    k = np.concatenate((O.apply_rope(k[..., :rot], inv, dtype), k[..., rot:]), -1)
    return q, k


CASES = [(2, 300, 4, 2, 256, 0.25, 1), (3, 70, 2, 1, 64, 1.0, 2), (1, 4096, 2, 1, 256, 1.0, 3)]


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_noalloc_matches_allocating_entry_point_twice(dtype):
    import torch

    lib = _lib.load()
    for b, s, hq, hkv, d, prf, seed in CASES:  # calls in a row, each with a different table
        qkv, qw, kw = _inputs(dtype, b, s, hq, hkv, d, seed)
        QW, KW = _device(qw, dtype), _device(kw, dtype)
        ref, got = _device(qkv, dtype), _device(qkv, dtype)
        _run(lib.clef_op_qk_norm_rope, dtype, ref, b, s, hq, hkv, d, prf, QW, KW)
        _run(lib.clef_op_qk_norm_rope_noalloc, dtype, got, b, s, hq, hkv, d, prf, QW, KW)
        torch.cuda.synchronize()
        got_h, ref_h = got.float().cpu().numpy(), ref.float().cpu().numpy()
        np.testing.assert_array_equal(got_h, ref_h)
        # Against the restatement at positions below 512.  The oracle's inverse
        # frequencies (NumPy's float32 power) and the library's (the host powf)
        # may differ in their last bit (2^-23 relative), so the float32 angle
        # at position p may differ by up to p x 2^-23 rad and a rotated value
        # of magnitude up to ~8 by p 2^-20: the FP32 tolerance allows that;
        # further out the bit-identical comparison above covers the table.
        p = min(s, 512)
        q, k = _oracle(qkv.reshape(b, s, -1)[:, :p].reshape(b * p, -1), b, p, hq, hkv, d, prf, qw, kw, dtype)
        x = got_h.reshape(b, s, -1)[:, :p]
        tol = dict(rtol=2 * 2.0**-7, atol=1e-2) if dtype == "bf16" else dict(rtol=1e-5, atol=1e-5 + p * 2.0**-20)
        np.testing.assert_allclose(x[..., : hq * 2 * d].reshape(b, p, hq, 2 * d)[..., :d], q, **tol)
        np.testing.assert_allclose(x[..., hq * 2 * d : hq * 2 * d + hkv * d].reshape(b, p, hkv, d), k, **tol)


def test_noalloc_rejects_sizes_beyond_its_table():
    lib = _lib.load()
    # s * rot/2 = 16385 * 64 > 1048576 entries: refused before any device work.
    st = lib.clef_op_qk_norm_rope_noalloc(_lib.DTYPE_BF16, 16, 1, 16385, 1, 1, 128, 1.0, 10000.0, 16, 16, 1e-6, None)
    assert st == _lib.CLEF_EINVAL
    assert b"exceeds" in lib.clef_last_error(None)
    # head_dim 2048 at partial rotary 1/16 (rot/2 = 64): its staged rows exceed 48 KB of shared memory
    st = lib.clef_op_qk_norm_rope_noalloc(_lib.DTYPE_BF16, 16, 1, 8, 1, 1, 2048, 1.0 / 16, 10000.0, 16, 16, 1e-6, None)
    assert st == _lib.CLEF_EINVAL
    assert b"1536" in lib.clef_last_error(None)
