"""The exact CUDA-core forward on shapes the tensor-core kernel does not take (needs a GPU).

``sdpa_exact_rt_kernel`` (csrc/fwd_exact.cu) serves every fp32 call and every
fp16 call the tensor-core kernel does not take, with E, Ev <= 128: odd head
dimensions (rows that are not whole 16-byte chunks take the converting loads
instead of cp.async), Ev != E, broadcast boolean and additive masks with any
strides, causal with L != S (top-left aligned), grouped-query heads, rows and
keys that are not multiples of its 64-row / 64-key tiles, fully-masked rows.
Each case is compared with the float64 oracle (``reference.py:56-163``) on
seeded inputs: fp32 at north_star's bound (rtol 1e-5, atol 1e-6 * max|v|),
fp16 at the conformance kit's 2e-3 with exact-zero dead rows.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle.sdpa import reference_sdpa

pytestmark = pytest.mark.gpu

# (lead q, lead kv, L, S, E, Ev, kwargs builder)
SHAPES = [
    ((2, 3), (2, 3), 70, 130, 33, 17, {}),
    ((1, 4), (1, 4), 64, 64, 128, 128, {"is_causal": True}),
    ((3,), (3,), 129, 65, 100, 96, {"is_causal": True}),       # L > S, causal top-left
    ((2, 6), (2, 2), 50, 200, 64, 64, {"enable_gqa": True}),
    ((2, 4), (2, 4), 97, 131, 64, 32, {"mask": "bool"}),
    ((2, 4), (2, 4), 40, 300, 8, 4, {"mask": "add"}),
    ((1, 2), (1, 2), 65, 129, 127, 128, {"mask": "bool_dead"}),
    ((4,), (4,), 1, 513, 64, 64, {}),
]


def _case(i, lq, lkv, L, S, E, Ev, spec, dtype):
    rng = np.random.default_rng(500 + i)
    q = rng.standard_normal(lq + (L, E)).astype(dtype)
    k = rng.standard_normal(lkv + (S, E)).astype(dtype)
    v = rng.standard_normal(lkv + (S, Ev)).astype(dtype)
    kw = {key: val for key, val in spec.items() if key != "mask"}
    m = spec.get("mask")
    if m in ("bool", "bool_dead"):
        mask = rng.random((lq[0], 1, L, S)) > 0.4          # broadcast over heads
        if m == "bool_dead":
            mask[:, :, 3, :] = False                        # a fully-masked row
            mask[:, :, :, 64:128] = False                   # a whole dead key tile
        kw["attn_mask"] = mask
    elif m == "add":
        kw["attn_mask"] = rng.standard_normal((L, S)).astype(np.float32)   # broadcast over lead
    return q, k, v, kw


@pytest.mark.parametrize("i", range(len(SHAPES)))
def test_exact_fp32_against_oracle(cuda_backend, i):
    lq, lkv, L, S, E, Ev, spec = SHAPES[i]
    q, k, v, kw = _case(i, lq, lkv, L, S, E, Ev, spec, np.float32)
    got = cuda_backend(q, k, v, **kw)
    want = reference_sdpa(q, k, v, **kw)
    assert got.dtype == np.float32 and got.shape == want.shape
    atol = 1e-6 * float(np.max(np.abs(v)))
    np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=1e-5, atol=atol)
    dead = np.all(want == 0, axis=-1)
    assert np.array_equal(got[dead], want[dead])


@pytest.mark.parametrize("i", [0, 2, 4, 5, 6])
def test_exact_fp16_against_oracle(cuda_backend, i):
    lq, lkv, L, S, E, Ev, spec = SHAPES[i]
    q, k, v, kw = _case(i, lq, lkv, L, S, E, Ev, spec, np.float16)
    got = cuda_backend(q, k, v, **kw)
    want = reference_sdpa(q, k, v, **kw)
    assert got.dtype == np.float16
    np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=2e-3, atol=2e-3)
    dead = np.all(want == 0, axis=-1)
    assert np.array_equal(got[dead], want[dead])
