"""The ``cuda`` SdpaBackend: NumPy in, NumPy out, computed on a B200.

:func:`scaled_dot_product_attention` has exactly the signature and error
contract of the reference backends (``src/portable_attention/dispatch.py:53-76``,
``src/portable_attention/reference.py:56-128``), so it registers with
``portable_attention.register_backend`` and passes the reference's conformance
kit unchanged. Each call validates, plans the descriptor, copies the operands
to the device, runs ``pa_sdpa_fwd`` (or ``pa_decode_fwd`` for length-1
queries) and copies the result back as a new array of ``query.dtype``; inputs
are never mutated. There is no CPU fallback: without the native library or a
GPU the call raises.

:func:`sdpa_device` is the same operation on device-resident buffers, for
callers that keep tensors on the GPU and time the kernels alone.
"""

from __future__ import annotations

import ctypes
import threading

import numpy as np

from ._lib import PA_MASK_NONE, check, lib
from .device import DeviceArena, Stream, sync_device_status
from .plan import plan_call
from .validation import validate

__all__ = ["scaled_dot_product_attention", "sdpa_device", "use_decode_kernel"]

_state = threading.local()
_arenas: dict[int, DeviceArena] = {}
_arena_lock = threading.Lock()


def _stream() -> Stream:
    s = getattr(_state, "stream", None)
    if s is None:
        s = Stream()
        _state.stream = s
    return s


def _arena() -> DeviceArena:
    dev = ctypes.c_int32(0)
    check(lib().pa_get_device(ctypes.byref(dev)))
    with _arena_lock:
        a = _arenas.get(dev.value)
        if a is None:
            a = _arenas[dev.value] = DeviceArena()
    return a


def use_decode_kernel(plan) -> bool:
    """Length-1 fp16 queries over dense (B, H, S, D) key/value go to split-KV decode.

    The decode kernel serves grouped-query groups of 1, 2, 4 or 8 query heads
    per key/value head; other groups take the tensor-core forward.
    """
    d = plan.desc
    return (plan.group in (1, 2, 4, 8) and plan.L == 1 and plan.cdt == np.float16 and plan.E == plan.Ev and plan.E in (64, 128)
            and plan.mask_kind == PA_MASK_NONE and not d.is_causal and plan.S >= 1
            and len(plan.out_lead) >= 1 and _dense_decode(plan))


def _dense_decode(plan) -> bool:
    d = plan.desc
    n = len(plan.out_lead)
    exp_q = plan.E
    exp_k = plan.S * plan.E
    for i in range(n - 1, -1, -1):
        dim = plan.out_lead[i]
        kdim = dim // plan.group if i == n - 1 else dim
        if dim > 1 and d.q_lead_stride[i] != exp_q:
            return False
        if kdim > 1 and (d.k_lead_stride[i] != exp_k or d.v_lead_stride[i] != exp_k):
            return False
        exp_q *= dim
        exp_k *= kdim
    return True


def scaled_dot_product_attention(query, key, value, attn_mask=None, dropout_p=0.0,
                                 is_causal=False, *, scale=None, enable_gqa=False):
    """SDPA on the GPU with the reference backend contract; returns ``query.dtype``."""
    group = validate(query, key, value, attn_mask, dropout_p, is_causal, enable_gqa)
    plan = plan_call(query.shape, key.shape, value.shape, query.dtype, key.dtype, value.dtype,
                     None if attn_mask is None else np.shape(attn_mask),
                     None if attn_mask is None else np.asarray(attn_mask).dtype,
                     is_causal, scale, group)
    cdt = plan.cdt
    host = [np.ascontiguousarray(x, dtype=cdt) for x in (query, key, value)]
    mask = None
    if plan.mask_kind != PA_MASK_NONE:
        mask = np.ascontiguousarray(np.asarray(attn_mask).reshape(plan.mask_shape),
                                    dtype=plan.mask_host_dtype)
    out = np.empty(plan.out_shape, dtype=cdt)
    if out.size == 0:
        return out.astype(query.dtype, copy=False)
    sizes = [a.nbytes for a in host] + [mask.nbytes if mask is not None else 0, out.nbytes]
    st = _stream()
    L = lib()
    arena = _arena()
    with arena.lock:
        dq, dk, dv, dm, do = arena.carve(sizes)
        for dptr, a in zip((dq, dk, dv), host):
            check(L.pa_memcpy_h2d(dptr, a.ctypes.data, a.nbytes, st.handle))
        if mask is not None:
            check(L.pa_memcpy_h2d(dm, mask.ctypes.data, mask.nbytes, st.handle))
        if use_decode_kernel(plan):
            check(L.pa_decode_fwd(ctypes.byref(plan.desc), dq, dk, dv, do, None, None, 0, st.handle))
        else:
            check(L.pa_sdpa_fwd(ctypes.byref(plan.desc), dq, dk, dv, dm if mask is not None else None,
                                do, None, st.handle))
        check(L.pa_memcpy_d2h(out.ctypes.data, do, out.nbytes, st.handle))
        st.synchronize()
    sync_device_status()
    return out.astype(query.dtype, copy=False)


def sdpa_device(plan, q_ptr, k_ptr, v_ptr, out_ptr, *, mask_ptr=None, lse_ptr=None,
                stream: Stream | None = None, decode=None, workspace=(None, 0)):
    """Launch the forward on device pointers described by ``plan`` (no sync, no copies)."""
    L = lib()
    handle = stream.handle if stream is not None else None
    if decode is None:
        decode = use_decode_kernel(plan)
    if decode:
        check(L.pa_decode_fwd(ctypes.byref(plan.desc), q_ptr, k_ptr, v_ptr, out_ptr, lse_ptr,
                              workspace[0], workspace[1], handle))
    else:
        check(L.pa_sdpa_fwd(ctypes.byref(plan.desc), q_ptr, k_ptr, v_ptr, mask_ptr, out_ptr,
                            lse_ptr, handle))
