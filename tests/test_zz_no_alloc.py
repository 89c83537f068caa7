"""The allocation-free q/k-norm + RoPE entry point against the allocating one.

``clef_op_qk_norm_rope_noalloc`` serves callers that cannot allocate device
memory (a framework that owns all device buffers, or a loop that must avoid
cudaMalloc's device synchronisation); it keeps its cos/sin tables in a fixed
array inside the library.  This file is named so pytest collects it last.
Each test runs two calls in a row with different shapes, so a table left
behind by the first call cannot satisfy the second.
"""

from __future__ import annotations

import numpy as np
import pytest

from deciax_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(dtype, b, s, hq, hkv, d, seed):
    import torch

    rng = np.random.default_rng(seed)
    n = hq * 2 * d + 2 * hkv * d
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    qkv = torch.from_numpy(rng.standard_normal((b * s, n)).astype(np.float32)).cuda().to(tdt)
    qw = torch.from_numpy(rng.standard_normal(d).astype(np.float32) * np.float32(0.1)).cuda().to(tdt)
    kw = torch.from_numpy(rng.standard_normal(d).astype(np.float32) * np.float32(0.1)).cuda().to(tdt)
    return qkv, qw, kw


def _run(fn, dtype, qkv, b, s, hq, hkv, d, prf, qw, kw):
    code = _lib.DTYPE_BF16 if dtype == "bf16" else _lib.DTYPE_F32
    st = fn(code, qkv.data_ptr(), b, s, hq, hkv, d, prf, 10000.0, qw.data_ptr(), kw.data_ptr(), 1e-6, None)
    _lib.check(st)


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_noalloc_matches_allocating_entry_point_twice(dtype):
    import torch

    lib = _lib.load()
    cases = [(2, 300, 4, 2, 256, 0.25, 1), (3, 70, 2, 1, 64, 1.0, 2)]  # two calls in a row, different tables
    for b, s, hq, hkv, d, prf, seed in cases:
        qkv, qw, kw = _inputs(dtype, b, s, hq, hkv, d, seed)
        ref = qkv.clone()
        _run(lib.clef_op_qk_norm_rope, dtype, ref, b, s, hq, hkv, d, prf, qw, kw)
        _run(lib.clef_op_qk_norm_rope_noalloc, dtype, qkv, b, s, hq, hkv, d, prf, qw, kw)
        torch.cuda.synchronize()
        got, want = qkv.float().cpu().numpy(), ref.float().cpu().numpy()
        tol = dict(rtol=2 * 2.0**-7, atol=1e-2) if dtype == "bf16" else dict(rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(got, want, **tol)


def test_noalloc_rejects_sizes_beyond_its_table():
    lib = _lib.load()
    # s * rot/2 = 16385 * 64 > 1048576 entries: refused before any device work.
    st = lib.clef_op_qk_norm_rope_noalloc(_lib.DTYPE_BF16, 16, 1, 16385, 1, 1, 128, 1.0, 10000.0, 16, 16, 1e-6, None)
    assert st == _lib.CLEF_EINVAL
    assert b"exceeds" in lib.clef_last_error(None)
