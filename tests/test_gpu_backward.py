"""Backward (VJP) parity on the GPU against the float64 oracle VJP.

The oracle VJP (``oracle/vjp.py``) is itself pinned by central finite
differences in ``tests/test_oracle.py``. Tolerance (fp16 inputs, fp32
accumulation): relative Frobenius error <= 2e-2 per gradient tensor, plus an
element-wise bound. At the full long-context size (q,k,v (1,32,131072,128))
the gradients are checked on sampled query rows and trailing key columns
against the oracle, and through exact identities of the VJP:
  sum_j dV_j = sum_i dO_i (per KV head, over its query-head group),
  sum_j dK_j = 0 (rows of dS sum to zero),
  sum(dQ * Q) = sum(dK * K) (both equal scale * sum dS * Q K^T).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle.sdpa import reference_lse, reference_sdpa
from oracle.vjp import reference_vjp

pytestmark = pytest.mark.gpu


def _rel(got, want):
    return float(np.linalg.norm(got.astype(np.float64) - want) / max(np.linalg.norm(want), 1e-30))


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", [(1, 2, 2, 128, 128), (2, 4, 2, 200, 333), (1, 8, 2, 300, 130),
                                   (1, 2, 1, 1, 77)], ids=["square", "gqa-ragged", "gqa-L>S", "one-row"])
def test_backward_matches_oracle(hd, causal, shape):
    import pa_b200

    b, hq, hkv, L, S = shape
    rng = np.random.default_rng(hd + 7 * causal + L)
    q = rng.standard_normal((b, hq, L, hd)).astype(np.float16)
    k = rng.standard_normal((b, hkv, S, hd)).astype(np.float16)
    v = rng.standard_normal((b, hkv, S, hd)).astype(np.float16)
    do = rng.standard_normal((b, hq, L, hd)).astype(np.float16)
    gqa = hq != hkv
    dq, dk, dv = pa_b200.sdpa_backward(q, k, v, do, is_causal=causal, enable_gqa=gqa)
    wq, wk, wv = reference_vjp(q, k, v, do, is_causal=causal, enable_gqa=gqa)
    for name, g, w in (("dq", dq, wq), ("dk", dk, wk), ("dv", dv, wv)):
        assert g.shape == w.shape and g.dtype == np.float16
        assert np.all(np.isfinite(g)), name
        # Relative Frobenius bound, with an absolute floor for gradients that
        # are exactly zero in exact arithmetic (a single causal row: dQ = 0).
        err = float(np.linalg.norm(g.astype(np.float64) - w))
        assert err <= 2e-2 * np.linalg.norm(w) + 1e-4 * np.sqrt(w.size), (name, err)
        np.testing.assert_allclose(g.astype(np.float64), w, rtol=5e-2, atol=2e-2 * np.abs(w).max() + 1e-4,
                                   err_msg=name)


def test_forward_lse_matches_oracle():
    import pa_b200

    rng = np.random.default_rng(4)
    q = rng.standard_normal((2, 4, 300, 128)).astype(np.float16)
    k = rng.standard_normal((2, 2, 300, 128)).astype(np.float16)
    v = rng.standard_normal((2, 2, 300, 128)).astype(np.float16)
    out, lse = pa_b200.forward_with_lse(q, k, v, is_causal=True, enable_gqa=True)
    np.testing.assert_allclose(out.astype(np.float64),
                               reference_sdpa(q, k, v, is_causal=True, enable_gqa=True),
                               rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(lse, reference_lse(q, k, is_causal=True, enable_gqa=True),
                               rtol=1e-4, atol=1e-3)


def test_backward_rejects_unsupported():
    import pa_b200

    z = np.zeros((1, 2, 8, 32), np.float16)
    with pytest.raises(NotImplementedError):
        pa_b200.sdpa_backward(z, z, z, z)  # head dim 32
    z = np.zeros((1, 2, 8, 64), np.float32)
    with pytest.raises(NotImplementedError):
        pa_b200.sdpa_backward(z, z, z, z)  # fp32
    z = np.zeros((1, 2, 8, 64), np.float16)
    with pytest.raises(NotImplementedError):
        pa_b200.sdpa_backward(z, z, z, z, attn_mask=np.ones((8, 8), bool))
    with pytest.raises(NotImplementedError, match="dropout_p"):
        pa_b200.sdpa_backward(z, z, z, z, dropout_p=0.1)


def _rows_oracle(q, k, v, do, rows, scale):
    """f64 dQ rows for causal attention of one head: needs only those rows' full softmax."""
    out = []
    k64, v64 = k.astype(np.float64), v.astype(np.float64)
    for i in rows:
        s = (k64[: i + 1] @ q[i].astype(np.float64)) * scale
        p = np.exp(s - s.max())
        p /= p.sum()
        o = p @ v64[: i + 1]
        dp = v64[: i + 1] @ do[i].astype(np.float64)
        ds = p * (dp - do[i].astype(np.float64) @ o)
        out.append(scale * ds @ k64[: i + 1])
    return np.array(out)


def _cols_oracle(q, k, v, do, cols, scale):
    """f64 dK, dV for trailing key columns of one causal head (seen only by rows >= j)."""
    j0 = min(cols)
    L = q.shape[0]
    q64, k64, v64, do64 = (x.astype(np.float64) for x in (q[j0:], k, v, do[j0:]))
    s = q64 @ k64.T * scale
    s[np.arange(L - j0)[:, None] + j0 < np.arange(k.shape[0])[None, :]] = -np.inf
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    p /= p.sum(axis=1, keepdims=True)
    o = p @ v64
    dp = do64 @ v64.T
    ds = p * (dp - np.sum(do64 * o, axis=1, keepdims=True))
    dv = p.T @ do64
    dk = scale * ds.T @ q64
    return dk[cols], dv[cols]


def test_full_size_long_causal_backward():
    import pa_b200
    from pa_b200 import workloads

    x = workloads.make("fp16_long_causal")
    q, k, v, do = x["q"], x["k"], x["v"], x["dout"]
    dq, dk, dv = pa_b200.sdpa_backward(q, k, v, do, is_causal=True)
    for g in (dq, dk, dv):
        assert np.all(np.isfinite(g))
    scale = 1 / np.sqrt(128)
    S = q.shape[2]
    for h in (0, 17, 31):
        rows = [0, 1, 4095, 70000, S - 1]
        want = _rows_oracle(q[0, h], k[0, h], v[0, h], do[0, h], rows, scale)
        got = dq[0, h, rows].astype(np.float64)
        assert _rel(got, want) <= 2e-2, (h, _rel(got, want))
        cols = [S - 64, S - 33, S - 2, S - 1]
        wk, wv = _cols_oracle(q[0, h], k[0, h], v[0, h], do[0, h], cols, scale)
        assert _rel(dk[0, h, cols], wk) <= 2e-2 and _rel(dv[0, h, cols], wv) <= 2e-2
    # Identities of the VJP over the whole tensors, bounded by L1 norms (the
    # sums cancel, so a relative bound on the sums themselves would be vacuous).
    dv64, do64 = dv.astype(np.float64), do.astype(np.float64)
    assert np.all(np.abs(dv64.sum(axis=2) - do64.sum(axis=2)) <= 2e-3 * np.abs(do64).sum(axis=2))
    del dv64, do64
    dk64 = dk.astype(np.float64)
    assert np.all(np.abs(dk64.sum(axis=2)) <= 2e-3 * np.abs(dk64).sum(axis=2) + 1e-3)
    qk = dk64 * k.astype(np.float64)
    rhs, rhs_l1 = float(qk.sum()), float(np.abs(qk).sum())
    del dk64, qk
    qq = dq.astype(np.float64) * q.astype(np.float64)
    lhs, lhs_l1 = float(qq.sum()), float(np.abs(qq).sum())
    assert abs(lhs - rhs) <= 1e-3 * (lhs_l1 + rhs_l1)
