"""bf16 operands through the C ABI (NumPy has no bfloat16, so the tests hold
bf16 values as uint16 bit patterns and hand the library a bf16 descriptor).

Inputs are rounded to bf16 (nearest-even) and the float64 oracle runs on the
exactly-representable rounded values. bf16 keeps 8 significand bits, so the
tolerance is max-abs 1.6e-2 / rel 1e-2 on outputs (4x the bf16 spacing at 1)
and 3e-2 relative Frobenius on gradients.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle.sdpa import reference_lse, reference_sdpa
from oracle.vjp import reference_vjp

pytestmark = pytest.mark.gpu


def to_bf16_bits(x):
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    b = b + 0x7FFF + ((b >> 16) & 1)          # round to nearest even
    return (b >> 16).astype(np.uint16)


def from_bf16_bits(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def _bf16_plan(q, k, v, **kw):
    import pa_b200
    from pa_b200._lib import PA_BF16

    group = q.shape[1] // k.shape[1]
    plan = pa_b200.plan_call(q.shape, k.shape, v.shape, np.float16, np.float16, np.float16,
                             group=group, **kw)
    plan.desc.dtype = PA_BF16
    return plan


def _upload(st, *arrays):
    from pa_b200._lib import check, lib
    from pa_b200.device import DeviceBuffer

    bufs = []
    for a in arrays:
        b = DeviceBuffer(a.nbytes)
        check(lib().pa_memcpy_h2d(b.ptr, a.ctypes.data, a.nbytes, st.handle))
        bufs.append(b)
    return bufs


def _download(st, buf, shape, dtype):
    from pa_b200._lib import check, lib

    out = np.empty(shape, dtype)
    check(lib().pa_memcpy_d2h(out.ctypes.data, buf.ptr, out.nbytes, st.handle))
    return out


@pytest.mark.parametrize("hd,causal,shape", [(128, True, (2, 8, 2, 300, 300)), (64, False, (1, 4, 4, 200, 333)),
                                             (128, False, (1, 4, 1, 1, 5000)),
                                             # head dim 40: the exact CUDA-core kernel's bf16 path
                                             (40, True, (1, 4, 2, 100, 130)), (40, False, (2, 4, 4, 1, 300))])
def test_bf16_forward_and_decode(hd, causal, shape):
    import pa_b200
    from pa_b200._lib import check, lib
    from pa_b200.backend import use_decode_kernel
    from pa_b200.device import DeviceBuffer, Stream

    b, hq, hkv, L, S = shape
    rng = np.random.default_rng(hd + L)
    qb, kb, vb = (to_bf16_bits(rng.standard_normal(s)) for s in
                  ((b, hq, L, hd), (b, hkv, S, hd), (b, hkv, S, hd)))
    q, k, v = (from_bf16_bits(x) for x in (qb, kb, vb))
    plan = _bf16_plan(qb, kb, vb, is_causal=causal)
    st = Stream()
    dq, dk, dv = _upload(st, qb, kb, vb)
    out = DeviceBuffer(qb.nbytes)
    lse = DeviceBuffer(b * hq * L * 4)
    if use_decode_kernel(plan):
        check(lib().pa_decode_fwd(ctypes.byref(plan.desc), dq.ptr, dk.ptr, dv.ptr, out.ptr, lse.ptr,
                                  None, 0, st.handle))
    else:
        check(lib().pa_sdpa_fwd(ctypes.byref(plan.desc), dq.ptr, dk.ptr, dv.ptr, None, out.ptr,
                                lse.ptr, st.handle))
    got = from_bf16_bits(_download(st, out, qb.shape, np.uint16))
    got_lse = _download(st, lse, (b, hq, L), np.float32)
    st.synchronize()
    pa_b200.sync_device_status()
    want = reference_sdpa(q, k, v, is_causal=causal, enable_gqa=hq != hkv)
    np.testing.assert_allclose(got.astype(np.float64), want, rtol=1e-2, atol=1.6e-2)
    np.testing.assert_allclose(got_lse, reference_lse(q, k, is_causal=causal, enable_gqa=hq != hkv),
                               rtol=1e-4, atol=2e-3)


def test_bf16_backward():
    import pa_b200
    from pa_b200._lib import check, lib
    from pa_b200.device import DeviceBuffer, Stream

    rng = np.random.default_rng(21)
    shapes = ((1, 4, 256, 128), (1, 2, 256, 128), (1, 2, 256, 128), (1, 4, 256, 128))
    qb, kb, vb, dob = (to_bf16_bits(rng.standard_normal(s)) for s in shapes)
    q, k, v, do = (from_bf16_bits(x) for x in (qb, kb, vb, dob))
    plan = _bf16_plan(qb, kb, vb, is_causal=True)
    st = Stream()
    dq_, dk_, dv_, ddo = _upload(st, qb, kb, vb, dob)
    out, lse = DeviceBuffer(qb.nbytes), DeviceBuffer(4 * 256 * 4)
    gq, gk, gv = DeviceBuffer(qb.nbytes), DeviceBuffer(kb.nbytes), DeviceBuffer(vb.nbytes)
    d = ctypes.byref(plan.desc)
    check(lib().pa_sdpa_fwd(d, dq_.ptr, dk_.ptr, dv_.ptr, None, out.ptr, lse.ptr, st.handle))
    check(lib().pa_sdpa_bwd(d, dq_.ptr, dk_.ptr, dv_.ptr, out.ptr, ddo.ptr, lse.ptr, gq.ptr, gk.ptr,
                            gv.ptr, st.handle))
    got = [from_bf16_bits(_download(st, g, s, np.uint16)) for g, s in
           ((gq, qb.shape), (gk, kb.shape), (gv, vb.shape))]
    st.synchronize()
    pa_b200.sync_device_status()
    want = reference_vjp(q, k, v, do, is_causal=True, enable_gqa=True)
    for name, g, w in zip(("dq", "dk", "dv"), got, want):
        rel = np.linalg.norm(g.astype(np.float64) - w) / np.linalg.norm(w)
        assert rel <= 3e-2, (name, rel)
