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
import os
import threading

import numpy as np

from ._lib import PA_MASK_NONE, check, lib
from .device import DeviceArena, Event, Stream, is_pinned, pinned_empty, sync_device_status
from .plan import plan_call
from .validation import validate

__all__ = ["scaled_dot_product_attention", "sdpa_device", "sdpa_sharded", "use_decode_kernel"]

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

    The decode kernel serves grouped-query groups of 1 to 16 query heads per
    key/value head; larger groups take the tensor-core forward.
    """
    d = plan.desc
    return (1 <= plan.group <= 16 and plan.L == 1 and plan.cdt == np.float16 and plan.E == plan.Ev and plan.E in (64, 128)
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


_CHUNK_BYTES = 48 << 20   # target host<->device bytes per pipelined chunk
_PIPELINE_MIN = 64 << 20  # below this a call is not worth splitting
_PINNED_OUT_MIN = 1 << 20


class _Pipes(threading.local):
    """Per-thread streams for copy-in, compute and copy-out, and their events."""

    def __init__(self):
        self.h2d = self.d2h = None
        self.events = []

    def ensure(self, n_events):
        if self.h2d is None:
            self.h2d, self.d2h = Stream(), Stream()
        while len(self.events) < n_events:
            self.events.append((Event(), Event()))
        return self.h2d, self.d2h, self.events[:n_events]


_pipes = _Pipes()


def _chunks(plan, host, out_nbytes):
    """Split along leading dim 0 when every operand carries it densely."""
    d = plan.desc
    if not plan.out_lead or plan.out_lead[0] < 2:
        return 1
    if 0 in (d.q_lead_stride[0], d.k_lead_stride[0], d.v_lead_stride[0]):
        return 1
    total = sum(a.nbytes for a in host) + out_nbytes
    if total < _PIPELINE_MIN:
        return 1
    return int(min(plan.out_lead[0], max(2, total // _CHUNK_BYTES)))


def scaled_dot_product_attention(query, key, value, attn_mask=None, dropout_p=0.0,
                                 is_causal=False, *, scale=None, enable_gqa=False):
    """SDPA on the GPU with the reference backend contract; returns ``query.dtype``.

    Large calls are cut along the first leading dimension and pipelined over
    three streams, so the host->device copy of chunk c+1, the kernel of chunk
    c and the device->host copy of chunk c-1 overlap; the result lands in a
    page-locked array from the library's pool (plain NumPy array semantics).
    """
    group = validate(query, key, value, attn_mask, dropout_p, is_causal, enable_gqa)
    plan = plan_call(query.shape, key.shape, value.shape, query.dtype, key.dtype, value.dtype,
                     None if attn_mask is None else np.shape(attn_mask),
                     None if attn_mask is None else np.asarray(attn_mask).dtype,
                     is_causal, scale, group)
    cdt = plan.cdt
    host = [np.ascontiguousarray(x, dtype=cdt) for x in (query, key, value)]
    mask = None
    if plan.mask_kind != PA_MASK_NONE:
        m = np.asarray(attn_mask).reshape(plan.mask_shape)
        if m.dtype == np.bool_:
            mask = np.ascontiguousarray(m).view(np.uint8)  # same bytes, no conversion copy
        else:
            mask = np.ascontiguousarray(m, dtype=plan.mask_host_dtype)
    out_nbytes = int(np.prod(plan.out_shape)) * cdt.itemsize
    if out_nbytes >= _PINNED_OUT_MIN:
        out = pinned_empty(plan.out_shape, cdt)
    else:
        out = np.empty(plan.out_shape, dtype=cdt)
    if out.size == 0:
        return out.astype(query.dtype, copy=False)
    sizes = [a.nbytes for a in host] + [mask.nbytes if mask is not None else 0, out.nbytes]
    st = _stream()
    L = lib()
    decode = use_decode_kernel(plan)
    n_chunks = 1 if decode else _chunks(plan, host, out.nbytes)
    arena = _arena()
    with arena.lock:
        dq, dk, dv, dm, do = arena.carve(sizes)
        if n_chunks == 1:
            for dptr, a in zip((dq, dk, dv), host):
                check(L.pa_memcpy_h2d(dptr, a.ctypes.data, a.nbytes, st.handle))
            if mask is not None:
                check(L.pa_memcpy_h2d(dm, mask.ctypes.data, mask.nbytes, st.handle))
            if decode:
                check(L.pa_decode_fwd(ctypes.byref(plan.desc), dq, dk, dv, do, None, None, 0,
                                      st.handle))
            else:
                check(L.pa_sdpa_fwd(ctypes.byref(plan.desc), dq, dk, dv,
                                    dm if mask is not None else None, do, None, st.handle))
            check(L.pa_memcpy_d2h(out.ctypes.data, do, out.nbytes, st.handle))
            st.synchronize()
        else:
            _run_pipelined(plan, host, mask, out, (dq, dk, dv, dm, do), n_chunks, query, key,
                           value, attn_mask, is_causal, scale, group, st)
    sync_device_status()
    return out.astype(query.dtype, copy=False)


def sdpa_sharded(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, *, scale=None,
                 enable_gqa=False, devices=None):
    """The same call as :func:`scaled_dot_product_attention`, spread over several GPUs.

    The first leading dimension is cut into one contiguous shard per device
    (``devices``: CUDA device indices, default every visible device) through
    ``pa_shard_fwd``; each device copies in its rows, runs the same kernels
    and copies its rows of the result back, driven by its own host thread.
    Results are identical to the single-GPU call.
    """
    from .device import device_count

    group = validate(query, key, value, attn_mask, dropout_p, is_causal, enable_gqa)
    plan = plan_call(query.shape, key.shape, value.shape, query.dtype, key.dtype, value.dtype,
                     None if attn_mask is None else np.shape(attn_mask),
                     None if attn_mask is None else np.asarray(attn_mask).dtype,
                     is_causal, scale, group)
    cdt = plan.cdt
    host = [np.ascontiguousarray(x, dtype=cdt) for x in (query, key, value)]
    mask = None
    if plan.mask_kind != PA_MASK_NONE:
        m = np.asarray(attn_mask).reshape(plan.mask_shape)
        mask = (np.ascontiguousarray(m).view(np.uint8) if m.dtype == np.bool_
                else np.ascontiguousarray(m, dtype=plan.mask_host_dtype))
    out = np.empty(plan.out_shape, dtype=cdt)
    if out.size == 0:
        return out.astype(query.dtype, copy=False)
    devs = list(range(device_count())) if devices is None else [int(x) for x in devices]
    if not devs:
        raise ValueError("sdpa_sharded: no CUDA device to run on")
    arr = (ctypes.c_int32 * len(devs))(*devs)
    check(lib().pa_shard_fwd(len(devs), arr, ctypes.byref(plan.desc), host[0].ctypes.data,
                             host[1].ctypes.data, host[2].ctypes.data,
                             mask.ctypes.data if mask is not None else None, out.ctypes.data, None))
    return out.astype(query.dtype, copy=False)


_STAGE_THREADS = max(1, min(8, os.cpu_count() or 1))
_stage_pool = None
_stage_lock = threading.Lock()


def _stage_executor():
    global _stage_pool
    with _stage_lock:
        if _stage_pool is None:
            from concurrent.futures import ThreadPoolExecutor

            _stage_pool = ThreadPoolExecutor(_STAGE_THREADS, thread_name_prefix="pa_b200_stage")
    return _stage_pool


def _parallel_copy(dst: np.ndarray, src: np.ndarray) -> None:
    """dst[:] = src for flat uint8 views, split over the staging threads (NumPy
    releases the GIL for plain copies, so the parts run in parallel)."""
    n = src.nbytes
    parts = _STAGE_THREADS if n >= (8 << 20) else 1
    if parts == 1:
        np.copyto(dst, src)
        return
    step = (n + parts - 1) // parts
    futs = [_stage_executor().submit(np.copyto, dst[o:o + step], src[o:o + step])
            for o in range(0, n, step)]
    for f in futs:
        f.result()


def _run_pipelined(plan, host, mask, out, ptrs, n_chunks, query, key, value, attn_mask,
                   is_causal, scale, group, st):
    """Copy-in / compute / copy-out of batch chunks on three overlapping streams.

    Pageable inputs (ordinary NumPy arrays) are staged chunk by chunk into two
    page-locked buffers per operand by a parallel host copy, so the copy of
    chunk c+1 overlaps the DMA of chunk c; the driver's own staging of a
    pageable copy is several times slower than PCIe.
    """
    L = lib()
    h2d, d2h, events = _pipes.ensure(n_chunks)
    dq, dk, dv, dm, do = ptrs
    B = plan.out_lead[0]
    bounds = [(B * c) // n_chunks for c in range(n_chunks + 1)]
    per = [a.nbytes // B for a in host]
    stage = [None if is_pinned(a) else
             [pinned_empty((max(bounds[c + 1] - bounds[c] for c in range(n_chunks)) * n,), np.uint8)
              for _ in range(2)]
             for a, n in zip(host, per)]
    flat = [a.reshape(-1).view(np.uint8) for a in host]
    out_per = out.nbytes // B
    mask_split = mask is not None and plan.desc.m_lead_stride[0] != 0
    mask_per = mask.nbytes // B if mask_split else 0
    if mask is not None and not mask_split:
        check(L.pa_memcpy_h2d(dm, mask.ctypes.data, mask.nbytes, h2d.handle))
    ready = Event()
    ready.record(st)        # the arena's previous users are done with these buffers
    ready.wait_on(h2d)
    for c in range(n_chunks):
        b0, b1 = bounds[c], bounds[c + 1]
        loaded, computed = events[c]
        if c >= 2 and any(sg is not None for sg in stage):
            events[c - 2][0].synchronize()   # that chunk's copies out of its staging slot are done
        for i, (dptr, a, n) in enumerate(zip((dq, dk, dv), host, per)):
            nb = (b1 - b0) * n
            if stage[i] is None:
                check(L.pa_memcpy_h2d(dptr + b0 * n, a.ctypes.data + b0 * n, nb, h2d.handle))
            else:
                slot = stage[i][c & 1]
                _parallel_copy(slot[:nb], flat[i][b0 * n:b1 * n])
                check(L.pa_memcpy_h2d(dptr + b0 * n, slot.ctypes.data, nb, h2d.handle))
        if mask_split:
            check(L.pa_memcpy_h2d(dm + b0 * mask_per, mask.ctypes.data + b0 * mask_per,
                                  (b1 - b0) * mask_per, h2d.handle))
        loaded.record(h2d)
        loaded.wait_on(st)
        shp = lambda x: (b1 - b0,) + tuple(np.shape(x))[1:]  # noqa: E731
        m_shape = None
        if mask is not None:
            m_shape = shp(mask) if mask_split else mask.shape
        sub = plan_call(shp(query), shp(key), shp(value), query.dtype, key.dtype, value.dtype,
                        m_shape, None if mask is None else np.asarray(attn_mask).dtype,
                        is_causal, scale, group)
        m_ptr = None
        if mask is not None:
            m_ptr = dm + (b0 * mask_per if mask_split else 0)
        check(L.pa_sdpa_fwd(ctypes.byref(sub.desc), dq + b0 * per[0], dk + b0 * per[1],
                            dv + b0 * per[2], m_ptr, do + b0 * out_per, None, st.handle))
        computed.record(st)
        computed.wait_on(d2h)
        check(L.pa_memcpy_d2h(out.ctypes.data + b0 * out_per, do + b0 * out_per,
                              (b1 - b0) * out_per, d2h.handle))
    d2h.synchronize()
    st.synchronize()


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
