"""Forward parity of the CUDA backend (needs a B200 and libpa_b200.so).

Every comparison is against outputs the real reference produced
(``tests/golden``) or against the CPU oracle on the same seeded inputs:

* the 26-case conformance matrix, with the reference kit's own acceptance rule
  (shape, dtype, finiteness, per-dtype ``allclose``, exact-zero dead rows);
* extra edge cases (L != S causal alignment, broadcast / additive / dead-row
  masks, mixed dtypes, shapes the tensor-core and decode kernels take);
* sampled rows of the full-size workloads, plus size-independent properties
  of the whole output (finite, causal row 0 equals v[0], convex hull).

Tolerances: fp64 1e-11, fp32 rtol 1e-4 / atol 1e-5, fp16 2e-3 / 2e-3 -- the
conformance kit's (``src/portable_attention/conformance.py:66-70``); the fp16
rows of full-size workloads also meet max-abs 2e-3 / rel 1e-2.
"""

from __future__ import annotations

import numpy as np
import pytest

from extra_cases import extra_cases
from oracle import conformance as oc
from oracle.sdpa import reference_sdpa

pytestmark = pytest.mark.gpu

CASES = oc.cases()
TOL = {np.dtype(np.float64): (1e-11, 1e-11), np.dtype(np.float32): (1e-4, 1e-5),
       np.dtype(np.float16): (2e-3, 2e-3)}


@pytest.mark.parametrize("idx", range(len(CASES)), ids=[c.name for c in CASES])
def test_conformance_case(idx, cuda_backend, golden_conformance):
    ok, detail = oc.check(cuda_backend, CASES[idx], want=golden_conformance[f"{idx}_ref"])
    assert ok, detail


def test_reference_kit_runs_unchanged(cuda_backend, reference_package):
    """The reference's own kit (conformance.py:318 assert_conforms, :300 check_backend,
    :141 conformance_cases) on the CUDA backend, registered through register_backend."""
    pa = reference_package
    pa.assert_conforms(cuda_backend)
    results = pa.check_backend(cuda_backend, pa.conformance_cases())
    assert len(results) == 26 and all(r.passed for r in results)
    from portable_attention.dispatch import _REGISTRY

    saved = dict(_REGISTRY)
    try:
        import pa_b200

        assert pa_b200.register()
        assert "cuda" in pa.available_backends()
        pa.assert_conforms(pa.get_backend("cuda"))
    finally:
        _REGISTRY.clear()
        _REGISTRY.update(saved)


FP32_CASES = [i for i, c in enumerate(CASES) if np.dtype(c.dtype) == np.float32]


def _fp32_strict(got, want, v, what):
    """north_star's fp32 bound: rtol 1e-5, atol 1e-6 * max|v| (no looser)."""
    atol = 1e-6 * float(np.max(np.abs(v)))
    np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=1e-5,
                               atol=atol, err_msg=what)


@pytest.mark.parametrize("idx", FP32_CASES, ids=[CASES[i].name for i in FP32_CASES])
def test_fp32_conformance_within_1e5(idx, cuda_backend, golden_conformance):
    case = CASES[idx]
    q, k, v = case.inputs()
    got = cuda_backend(q, k, v, **case.kwargs)
    assert got.dtype == np.float32
    _fp32_strict(got, golden_conformance[f"{idx}_ref"], v, case.name)


def test_fp32_extra_cases_within_1e5(cuda_backend, golden_extra):
    seen = 0
    for i, (name, (q, k, v), kw) in enumerate(extra_cases()):
        if q.dtype != np.float32:
            continue
        _fp32_strict(cuda_backend(q, k, v, **kw), golden_extra[f"{i}_ref"], v, name)
        seen += 1
    assert seen


def test_fp32_workload_rows_within_1e5(cuda_backend, golden_rows):
    """The fp32 unmasked workload q,k,v (4, 8, 512, 64): golden rows at rtol 1e-5."""
    from pa_b200 import workloads

    x = workloads.make("fp32_unmasked")
    out = cuda_backend(x["q"], x["k"], x["v"])
    seen = 0
    for key, want in golden_rows.items():
        parts = key.split("|")
        if parts[0] != "fp32_unmasked" or parts[1] == "fingerprint":
            continue
        b, h, r0, nr = map(int, parts[1:])
        _fp32_strict(out[b, h, r0:r0 + nr], want, x["v"][b, h], key)
        seen += 1
    assert seen


def test_extra_cases(cuda_backend, golden_extra):
    failures = []
    for i, (name, (q, k, v), kw) in enumerate(extra_cases()):
        want = golden_extra[f"{i}_ref"]
        got = cuda_backend(q, k, v, **kw)
        assert got.dtype == q.dtype and got.shape == want.shape, name
        rtol, atol = TOL[q.dtype]
        if not np.allclose(got.astype(np.float64), want.astype(np.float64), rtol=rtol, atol=atol):
            failures.append(f"{name}: max abs {np.max(np.abs(got.astype(np.float64) - want)):.3e}")
        dead = np.all(want == 0, axis=-1)
        if np.any(dead) and not np.array_equal(got[dead], want[dead]):
            failures.append(f"{name}: dead rows not exactly zero")
    assert not failures, failures


def test_inputs_are_not_mutated(cuda_backend):
    rng = np.random.default_rng(5)
    q = rng.standard_normal((2, 4, 130, 64)).astype(np.float16)
    k = rng.standard_normal((2, 4, 200, 64)).astype(np.float16)
    v = rng.standard_normal((2, 4, 200, 64)).astype(np.float16)
    copies = [x.copy() for x in (q, k, v)]
    cuda_backend(q, k, v, is_causal=True)
    for a, b in zip((q, k, v), copies):
        np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
def test_tensor_core_path_random_shapes(cuda_backend, hd, causal):
    """Ragged L/S around the 128-row tile, GQA and causal, against the float64 oracle."""
    rng = np.random.default_rng(100 + hd + causal)
    for L, S, hq, hkv in ((1, 1, 2, 1), (127, 129, 4, 2), (256, 255, 2, 2), (383, 640, 8, 1)):
        q = rng.standard_normal((1, hq, L, hd)).astype(np.float16)
        k = rng.standard_normal((1, hkv, S, hd)).astype(np.float16)
        v = rng.standard_normal((1, hkv, S, hd)).astype(np.float16)
        got = cuda_backend(q, k, v, is_causal=causal, enable_gqa=hq != hkv)
        want = reference_sdpa(q, k, v, is_causal=causal, enable_gqa=hq != hkv)
        np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64),
                                   rtol=2e-3, atol=2e-3, err_msg=f"L={L} S={S}")


def test_large_logits_and_fully_masked_tiles(cuda_backend):
    """Scores far above the running max (rescale path) and whole masked key tiles."""
    rng = np.random.default_rng(7)
    q = (rng.standard_normal((1, 2, 256, 128)) * 4).astype(np.float16)
    k = (rng.standard_normal((1, 2, 512, 128)) * 4).astype(np.float16)
    v = rng.standard_normal((1, 2, 512, 128)).astype(np.float16)
    mask = np.ones((1, 1, 256, 512), dtype=bool)
    mask[..., 128:384] = False          # two whole key tiles masked
    mask[..., 5, :] = False             # one dead row
    got = cuda_backend(q, k, v, attn_mask=mask)
    want = reference_sdpa(q, k, v, attn_mask=mask)
    np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64), rtol=2e-3, atol=2e-3)
    assert np.all(got[..., 5, :] == 0)


def _check_rows(name, out, x, golden_rows, rtol, atol):
    group = x["q"].shape[1] // x["k"].shape[1]
    seen = 0
    for key, want in golden_rows.items():
        parts = key.split("|")
        if parts[0] != name or parts[1] == "fingerprint":
            continue
        b, h, r0, nr = map(int, parts[1:])
        got = out[b, h, r0:r0 + nr].astype(np.float64)
        w = want.astype(np.float64)
        np.testing.assert_allclose(got, w, rtol=rtol, atol=atol, err_msg=key)
        if out.dtype == np.float16:
            assert np.max(np.abs(got - w)) <= 2e-3, key
        seen += 1
    assert seen
    del group


@pytest.mark.parametrize("name", ["fp32_unmasked", "fp16_causal_gqa", "fp16_masked_cross"])
def test_full_size_workload_rows(cuda_backend, golden_rows, name):
    from pa_b200 import workloads

    w = workloads.WORKLOADS[name]
    x = workloads.make(name)
    fp = np.array([x["q"].ravel()[:4].astype(np.float64), x["k"].ravel()[-4:].astype(np.float64),
                   x["v"].ravel()[-4:].astype(np.float64)])
    np.testing.assert_array_equal(fp, golden_rows[f"{name}|fingerprint"])
    out = cuda_backend(x["q"], x["k"], x["v"], attn_mask=x.get("mask"), is_causal=w.is_causal,
                       enable_gqa=w.enable_gqa)
    assert out.shape == x["q"].shape[:-1] + (x["v"].shape[-1],) and out.dtype == x["q"].dtype
    assert np.all(np.isfinite(out))
    rtol, atol = TOL[out.dtype]
    _check_rows(name, out, x, golden_rows, rtol, atol)
    group = w.q_shape[1] // w.kv_shape[1]
    if w.is_causal:
        # Row 0 sees key 0 only: its output is v[0] of the matching kv head.
        for b in (0, w.q_shape[0] - 1):
            for h in (0, w.q_shape[1] - 1):
                np.testing.assert_array_equal(out[b, h, 0], x["v"][b, h // group, 0])
    # Convex hull: every output lies within the per-column range of v.
    vmin = x["v"].min(axis=2).astype(np.float32)
    vmax = x["v"].max(axis=2).astype(np.float32)
    vmin = np.repeat(vmin, group, axis=1)[:, :, None, :]
    vmax = np.repeat(vmax, group, axis=1)[:, :, None, :]
    o = out.astype(np.float32)
    assert np.all(o >= vmin - 2e-3) and np.all(o <= vmax + 2e-3)


def test_pageable_and_page_locked_inputs_give_identical_results(cuda_backend):
    """Large calls stage pageable inputs through page-locked buffers themselves."""
    import pa_b200
    from pa_b200.device import is_pinned

    rng = np.random.default_rng(37)
    q = rng.standard_normal((6, 8, 2048, 128)).astype(np.float16)
    k = rng.standard_normal((6, 8, 2048, 128)).astype(np.float16)
    v = rng.standard_normal((6, 8, 2048, 128)).astype(np.float16)
    pinned = [pa_b200.pinned_empty(x.shape, x.dtype) for x in (q, k, v)]
    for dst, src in zip(pinned, (q, k, v)):
        dst[...] = src
    assert is_pinned(pinned[0]) and not is_pinned(q)
    a = cuda_backend(q, k, v, is_causal=True)
    b = cuda_backend(*pinned, is_causal=True)
    np.testing.assert_array_equal(a, b)
    want = reference_sdpa(q[:1, :2], k[:1, :2], v[:1, :2], is_causal=True)
    np.testing.assert_allclose(a[:1, :2].astype(np.float64), want.astype(np.float64), rtol=2e-3, atol=2e-3)


def test_large_call_pipelined_over_batch_chunks_is_bit_identical(cuda_backend):
    """A call above the pipelining threshold is cut into batch chunks (copy-in, compute
    and copy-out overlapped on three streams); every row must equal a single launch's."""
    import pa_b200

    rng = np.random.default_rng(31)
    q = rng.standard_normal((4, 16, 2048, 128)).astype(np.float16)
    k = rng.standard_normal((4, 4, 2048, 128)).astype(np.float16)
    v = rng.standard_normal((4, 4, 2048, 128)).astype(np.float16)
    got = cuda_backend(q, k, v, is_causal=True, enable_gqa=True)
    one = pa_b200.sdpa_sharded(q, k, v, is_causal=True, enable_gqa=True, devices=[0])
    np.testing.assert_array_equal(got, one)
