"""Precision of the tensor-core Gated DeltaNet passes' rounding points (CPU).

The BF16 passes (``csrc/gdn_tc.cuh``) evaluate the chunked rule of
``kernels/gdn/reference.py:40-92`` with TF32 operands and FP32 accumulation:
kk^T and qk^T exact on the bf16 values, then M = (q k^T dk^-1/2) * decay,
T diag(beta), q dk^-1/2, R = v - e^g (k S), V_new = T diag(beta) R,
K~ = k e^(g_C - g) and the stored state each rounded to TF32.  This test
replays exactly those rounding points in NumPy and bounds the result against a
float64 token-by-token recurrence (reference.py:24-37) on the same bf16
inputs, across decay regimes from fast to almost none.  The GPU tests compare
the kernels themselves with the oracle.
"""

import ml_dtypes
import numpy as np
import pytest

F32 = np.float32
C = 64


def bf16(x):
    return np.asarray(x, F32).astype(ml_dtypes.bfloat16).astype(F32)


def tf32(x):
    """Round to TF32 (10-bit mantissa, to nearest, ties away from zero), as cvt.rna.tf32.f32."""
    x = np.asarray(x, F32)
    r = ((x.view(np.uint32) + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(F32)
    return np.where(np.isfinite(x), r, x).astype(F32)


def recurrence_f64(q, k, v, g, beta):
    s, dk = q.shape
    state = np.zeros((dk, v.shape[1]))
    out = np.zeros((s, v.shape[1]))
    for t in range(s):
        state *= np.exp(np.float64(g[t]))
        delta = (v[t].astype(np.float64) - state.T @ k[t]) * beta[t]
        state += np.outer(k[t], delta)
        out[t] = state.T @ q[t]
    return out


def tensor_core_schedule(q, k, v, g, beta, qscale):
    s, dk = q.shape
    n, pad = -(-s // C), (-s) % C
    q, k, v, g, beta = (np.pad(x, [(0, pad)] + [(0, 0)] * (x.ndim - 1)) for x in (q, k, v, g, beta))
    state = np.zeros((dk, v.shape[1]), F32)
    out = np.zeros((n * C, v.shape[1]), F32)
    low = np.tril(np.ones((C, C), bool))
    strict = np.tril(low, -1)
    for i in range(n):
        sl = slice(i * C, (i + 1) * C)
        qi, ki, vi, bi = q[sl], k[sl], v[sl], beta[sl]
        gi = np.cumsum(g[sl], dtype=F32)
        es, ws = np.exp(gi).astype(F32), np.exp(gi[-1] - gi).astype(F32)
        with np.errstate(over="ignore"):
            decay = np.exp(np.where(low, gi[:, None] - gi[None, :], -np.inf)).astype(F32)
        a = np.where(strict, -((ki @ ki.T) * bi[:, None]) * decay, 0).astype(F32)
        t = np.linalg.inv(np.eye(C) - a.astype(np.float64)).astype(F32)
        t_beta = tf32(t * bi[None, :])
        m = np.where(low, tf32((qi @ ki.T) * F32(qscale) * decay), 0).astype(F32)
        k_state = (ki @ state).astype(F32)
        q_state = (tf32(qi * F32(qscale)) @ state).astype(F32)
        r = tf32(vi - es[:, None] * k_state)
        v_new = tf32(t_beta @ r)
        out[sl] = es[:, None] * q_state + (m @ v_new).astype(F32)
        k_tilde = tf32(ki * ws[:, None])
        state = tf32(state * np.exp(gi[-1]).astype(F32) + (k_tilde.T @ v_new).astype(F32))
    return out[:s]


@pytest.mark.parametrize("s,lo,hi", [(2048, 0.005, 0.3), (2048, 0.3, 1.0), (1024, 0.9, 1.0), (2048, 0.995, 1.0)])
def test_tensor_core_rounding_points_stay_far_inside_a_bf16_step(s, lo, hi):
    rng = np.random.default_rng(s + int(lo * 1000))
    dk = dv = 128
    qscale = dk**-0.5
    q = rng.standard_normal((s, dk))
    k = rng.standard_normal((s, dk))
    q = bf16(q / np.linalg.norm(q, axis=1, keepdims=True))
    k = bf16(k / np.linalg.norm(k, axis=1, keepdims=True))
    v = bf16(rng.standard_normal((s, dv)))
    g = np.log(rng.uniform(lo, hi, s)).astype(F32)
    beta = bf16(1 / (1 + np.exp(-rng.standard_normal(s))))
    expected = recurrence_f64(q.astype(np.float64) * qscale, k.astype(np.float64), v, g, beta)
    got = tensor_core_schedule(q, k, v, g, beta, qscale)
    err = np.abs(got - expected).max() / np.abs(expected).max()
    # the bf16 output rounding's relative step is 2^-8 = 3.9e-3
    assert err < 1.5e-3, err
