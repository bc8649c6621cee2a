"""Backward pass (VJP) of the SDPA forward on the GPU, NumPy in / NumPy out.

The reference has no backward: its roadmap lists an optional autograd hook
(``ROADMAP.md:57-58``). :func:`sdpa_backward` is that hook for this backend: the
gradient of ``scaled_dot_product_attention`` (``reference.py:56-163``) with
respect to query, key and value for a given output cotangent. It runs the
tensor-core forward once (to get the output and the per-row log-sum-exp)
and then ``pa_sdpa_bwd``; grouped-query key/value gradients are summed over
their query-head group, so ``dk`` / ``dv`` have the key / value shapes.

Scope: dense fp16 (B, H, L, D) operands with D in {64, 128}, causal or not,
no attn_mask and no dropout; anything else raises ``NotImplementedError``
rather than computing elsewhere.
"""

from __future__ import annotations

import ctypes

import numpy as np

from ._lib import PA_MASK_NONE, check, lib
from .backend import _arena, _stream
from .device import sync_device_status
from .plan import plan_call
from .validation import validate

__all__ = ["forward_with_lse", "sdpa_backward"]


def _plan_tc(query, key, value, attn_mask, dropout_p, is_causal, scale, enable_gqa):
    group = validate(query, key, value, attn_mask, dropout_p, is_causal, enable_gqa)
    if attn_mask is not None:
        raise NotImplementedError("sdpa_backward does not support attn_mask yet")
    plan = plan_call(query.shape, key.shape, value.shape, query.dtype, key.dtype, value.dtype,
                     None, None, is_causal, scale, group)
    if plan.cdt != np.float16 or plan.E != plan.Ev or plan.E not in (64, 128):
        raise NotImplementedError(
            "sdpa_backward supports float16 query/key/value with head dim 64 or 128")
    if query.ndim < 3:
        raise NotImplementedError("sdpa_backward needs a head axis: (*, H, L, D)")
    if plan.mask_kind != PA_MASK_NONE:
        raise NotImplementedError("sdpa_backward does not support attn_mask yet")
    return plan


def forward_with_lse(query, key, value, dropout_p=0.0, is_causal=False, *, scale=None,
                     enable_gqa=False):
    """Forward output and the natural-log lse per query row (float32, shape ``(*, L)``)."""
    plan = _plan_tc(query, key, value, None, dropout_p, is_causal, scale, enable_gqa)
    host = [np.ascontiguousarray(x, dtype=np.float16) for x in (query, key, value)]
    out = np.empty(plan.out_shape, np.float16)
    lse = np.empty(plan.out_shape[:-1], np.float32)
    st, L = _stream(), lib()
    arena = _arena()
    with arena.lock:
        dq_, dk_, dv_, do_, dl_ = arena.carve([a.nbytes for a in host] + [out.nbytes, lse.nbytes])
        for dptr, a in zip((dq_, dk_, dv_), host):
            check(L.pa_memcpy_h2d(dptr, a.ctypes.data, a.nbytes, st.handle))
        check(L.pa_sdpa_fwd(ctypes.byref(plan.desc), dq_, dk_, dv_, None, do_, dl_, st.handle))
        check(L.pa_memcpy_d2h(out.ctypes.data, do_, out.nbytes, st.handle))
        check(L.pa_memcpy_d2h(lse.ctypes.data, dl_, lse.nbytes, st.handle))
        st.synchronize()
    sync_device_status()
    return out, lse


def sdpa_backward(query, key, value, dout, attn_mask=None, dropout_p=0.0, is_causal=False, *,
                  scale=None, enable_gqa=False):
    """Return ``(dq, dk, dv)`` for cotangent ``dout`` of the forward with these arguments."""
    plan = _plan_tc(query, key, value, attn_mask, dropout_p, is_causal, scale, enable_gqa)
    if tuple(np.shape(dout)) != plan.out_shape:
        raise ValueError(f"dout shape {np.shape(dout)} != output shape {plan.out_shape}")
    host = [np.ascontiguousarray(x, dtype=np.float16) for x in (query, key, value, dout)]
    dq = np.empty(query.shape, np.float16)
    dk = np.empty(key.shape, np.float16)
    dv = np.empty(value.shape, np.float16)
    out_bytes = int(np.prod(plan.out_shape)) * 2
    lse_bytes = int(np.prod(plan.out_shape[:-1])) * 4
    st, L = _stream(), lib()
    arena = _arena()
    with arena.lock:
        ptrs = arena.carve([a.nbytes for a in host] + [out_bytes, lse_bytes, dq.nbytes, dk.nbytes,
                                                        dv.nbytes])
        pq, pk, pv, pdo, po, plse, pdq, pdk, pdv = ptrs
        for dptr, a in zip((pq, pk, pv, pdo), host):
            check(L.pa_memcpy_h2d(dptr, a.ctypes.data, a.nbytes, st.handle))
        check(L.pa_sdpa_fwd(ctypes.byref(plan.desc), pq, pk, pv, None, po, plse, st.handle))
        check(L.pa_sdpa_bwd(ctypes.byref(plan.desc), pq, pk, pv, po, pdo, plse, pdq, pdk, pdv,
                            st.handle))
        for arr, dptr in ((dq, pdq), (dk, pdk), (dv, pdv)):
            check(L.pa_memcpy_d2h(arr.ctypes.data, dptr, arr.nbytes, st.handle))
        st.synchronize()
    sync_device_status()
    return dq, dk, dv
