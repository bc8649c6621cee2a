"""Split-KV decode (query length 1) parity on the GPU.

Against the float64 oracle on seeded inputs, the golden reference rows of the
full-size decode workload (q (64,32,1,128), k/v (64,8,32768,128)), and the
explicit-workspace entry point. fp16 tolerance: 2e-3 abs / 2e-3 rel.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle.sdpa import reference_lse, reference_sdpa

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("hq,hkv", [(8, 8), (8, 4), (8, 2), (16, 2), (6, 2), (12, 2), (18, 2), (32, 2), (5, 5)])
def test_decode_matches_oracle(cuda_backend, hd, hq, hkv):
    rng = np.random.default_rng(hd * 100 + hq * 10 + hkv)
    for S in (1, 31, 33, 1000, 4099):
        q = rng.standard_normal((3, hq, 1, hd)).astype(np.float16)
        k = rng.standard_normal((3, hkv, S, hd)).astype(np.float16)
        v = rng.standard_normal((3, hkv, S, hd)).astype(np.float16)
        got = cuda_backend(q, k, v, enable_gqa=hq != hkv)
        want = reference_sdpa(q, k, v, enable_gqa=hq != hkv)
        np.testing.assert_allclose(got.astype(np.float64), want.astype(np.float64),
                                   rtol=2e-3, atol=2e-3, err_msg=f"S={S}")


def test_decode_routes_to_decode_kernel():
    import pa_b200
    from pa_b200.backend import use_decode_kernel

    plan = pa_b200.plan_call((64, 32, 1, 128), (64, 8, 32768, 128), (64, 8, 32768, 128),
                             np.float16, np.float16, np.float16, group=4)
    assert use_decode_kernel(plan)
    plan = pa_b200.plan_call((2, 6, 1, 128), (2, 2, 100, 128), (2, 2, 100, 128),
                             np.float16, np.float16, np.float16, group=3)
    assert use_decode_kernel(plan)  # any group of 1 to 16 query heads per key/value head
    plan = pa_b200.plan_call((2, 34, 1, 128), (2, 2, 100, 128), (2, 2, 100, 128),
                             np.float16, np.float16, np.float16, group=17)
    assert not use_decode_kernel(plan)  # a group of 17 takes the tensor-core forward


def test_decode_explicit_workspace_and_lse():
    import pa_b200
    from pa_b200._lib import check, lib
    from pa_b200.device import DeviceBuffer, Stream

    rng = np.random.default_rng(11)
    q = (rng.standard_normal((2, 8, 1, 128)) * 0.5).astype(np.float16)
    k = (rng.standard_normal((2, 2, 7000, 128)) * 0.5).astype(np.float16)
    v = (rng.standard_normal((2, 2, 7000, 128)) * 0.5).astype(np.float16)
    plan = pa_b200.plan_call(q.shape, k.shape, v.shape, q.dtype, k.dtype, v.dtype, group=4)
    need = ctypes.c_size_t(0)
    check(lib().pa_decode_workspace_size(ctypes.byref(plan.desc), ctypes.byref(need)))
    assert need.value > 0
    st = Stream()
    bufs = [DeviceBuffer(x.nbytes) for x in (q, k, v)]
    for b, x in zip(bufs, (q, k, v)):
        check(lib().pa_memcpy_h2d(b.ptr, x.ctypes.data, x.nbytes, st.handle))
    out = DeviceBuffer(q.nbytes)
    lse = DeviceBuffer(2 * 8 * 4)
    ws = DeviceBuffer(need.value)
    too_small = lib().pa_decode_fwd(ctypes.byref(plan.desc), bufs[0].ptr, bufs[1].ptr, bufs[2].ptr,
                                    out.ptr, lse.ptr, ws.ptr, need.value - 4, st.handle)
    assert too_small != 0
    check(lib().pa_decode_fwd(ctypes.byref(plan.desc), bufs[0].ptr, bufs[1].ptr, bufs[2].ptr,
                              out.ptr, lse.ptr, ws.ptr, need.value, st.handle))
    o = np.empty_like(q)
    l = np.empty((2, 8, 1), np.float32)
    check(lib().pa_memcpy_d2h(o.ctypes.data, out.ptr, o.nbytes, st.handle))
    check(lib().pa_memcpy_d2h(l.ctypes.data, lse.ptr, l.nbytes, st.handle))
    st.synchronize()
    pa_b200.sync_device_status()
    np.testing.assert_allclose(o.astype(np.float64), reference_sdpa(q, k, v, enable_gqa=True),
                               rtol=2e-3, atol=2e-3)
    np.testing.assert_allclose(l, reference_lse(q, k, enable_gqa=True), rtol=1e-4, atol=1e-4)


def test_full_size_decode_rows(cuda_backend, golden_rows):
    from pa_b200 import workloads

    x = workloads.make("fp16_decode_gqa")
    fp = np.array([x["q"].ravel()[:4].astype(np.float64), x["k"].ravel()[-4:].astype(np.float64),
                   x["v"].ravel()[-4:].astype(np.float64)])
    np.testing.assert_array_equal(fp, golden_rows["fp16_decode_gqa|fingerprint"])
    out = cuda_backend(x["q"], x["k"], x["v"], enable_gqa=True)
    assert out.shape == (64, 32, 1, 128) and out.dtype == np.float16
    assert np.all(np.isfinite(out))
    seen = 0
    for key, want in golden_rows.items():
        parts = key.split("|")
        if parts[0] != "fp16_decode_gqa" or parts[1] == "fingerprint":
            continue
        b, h, r0, nr = map(int, parts[1:])
        got = out[b, h, r0:r0 + nr].astype(np.float64)
        np.testing.assert_allclose(got, want.astype(np.float64), rtol=2e-3, atol=2e-3, err_msg=key)
        seen += 1
    assert seen == 5
    # Size-independent property: a weighted mean of |v| is bounded by max |v| per column.
    vmax = np.abs(x["v"]).max(axis=2).astype(np.float32)
    assert np.all(np.abs(out[:, :, 0].astype(np.float32)) <= np.repeat(vmax, 4, axis=1) + 2e-3)
