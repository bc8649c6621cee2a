"""Decode (query length 1) over a key/value cache: varlen, paged and fp8 e4m3.

The reference's SdpaBackend takes dense key/value tensors
(``src/portable_attention/dispatch.py:53-76``); a serving stack decodes from
a cache whose sequences have their own lengths, often split into pages named
by a block table and stored as fp8. These entry points run the same math
(``reference.py:139-162`` per sequence over its own keys) on such caches
through ``pa_decode_kv_fwd`` (include/pa_b200.h).

Cache layouts (``layout``):

* ``"hnd"`` -- ``(pages, kv_heads, page_size, head_dim)``
* ``"nhd"`` -- ``(pages, page_size, kv_heads, head_dim)``

Without a block table page ``b`` holds sequence ``b``, so a dense
``(batch, kv_heads, S, head_dim)`` cache is the ``"hnd"`` case with
``page_size = S``. fp8 caches are ``uint8`` arrays of e4m3 bit patterns with
``kv_format="e4m3"`` and per-tensor ``k_scale`` / ``v_scale``.

:func:`decode_kv_cache` takes NumPy arrays (copied to the device each call);
:func:`decode_kv_device` launches on device pointers (no copies, no sync).
"""

from __future__ import annotations

import ctypes
import math

import numpy as np

from ._lib import PA_BF16, PA_F16, PA_FP8_E4M3, KvCacheDesc, check, lib
from .device import Stream, sync_device_status

__all__ = ["decode_kv_cache", "decode_kv_device", "kv_cache_desc", "kv_workspace_size"]

_LAYOUTS = ("hnd", "nhd")


def kv_cache_desc(batch, q_heads, head_dim, cache_shape, *, layout="hnd", q_dtype="f16",
                  kv_format=None, paged=False, max_pages_per_seq=0, max_seq_len=None,
                  scale=None, k_scale=1.0, v_scale=1.0) -> KvCacheDesc:
    """Fill a ``pa_kv_cache_desc`` for a dense cache array of ``cache_shape`` in ``layout``."""
    if layout not in _LAYOUTS:
        raise ValueError(f"layout must be one of {_LAYOUTS}, got {layout!r}")
    if len(cache_shape) != 4:
        raise ValueError(f"cache must be 4-D (pages, ..., head_dim), got shape {tuple(cache_shape)}")
    pages, a1, a2, d = (int(x) for x in cache_shape)
    kv_heads, page_size = (a1, a2) if layout == "hnd" else (a2, a1)
    if d != head_dim:
        raise ValueError(f"cache head_dim {d} does not match the query's {head_dim}")
    if q_heads % kv_heads:
        raise ValueError(f"q_heads ({q_heads}) must be a multiple of kv_heads ({kv_heads})")
    desc = KvCacheDesc()
    desc.q_dtype = {"f16": PA_F16, "bf16": PA_BF16}[q_dtype]
    desc.kv_dtype = PA_FP8_E4M3 if kv_format == "e4m3" else desc.q_dtype
    desc.batch, desc.q_heads, desc.kv_heads, desc.head_dim = batch, q_heads, kv_heads, head_dim
    desc.page_size, desc.num_pages = page_size, pages
    desc.max_pages_per_seq = max_pages_per_seq if paged else 1
    if max_seq_len is None:
        max_seq_len = max_pages_per_seq * page_size if paged else page_size
    desc.max_seq_len = int(max_seq_len)
    if layout == "hnd":
        desc.key_stride, desc.head_stride = d, page_size * d
    else:
        desc.key_stride, desc.head_stride = kv_heads * d, d
    desc.page_stride = kv_heads * page_size * d
    desc.scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)
    desc.k_scale, desc.v_scale = float(k_scale), float(v_scale)
    return desc


def kv_workspace_size(desc: KvCacheDesc, paged: bool) -> int:
    n = ctypes.c_size_t(0)
    check(lib().pa_decode_kv_workspace_size(ctypes.byref(desc), int(bool(paged)), ctypes.byref(n)))
    return int(n.value)


def decode_kv_device(desc: KvCacheDesc, q_ptr, k_ptr, v_ptr, out_ptr, *, block_table_ptr=None,
                     seq_lens_ptr=None, lse_ptr=None, stream: Stream | None = None,
                     workspace=(None, 0)) -> None:
    """Launch ``pa_decode_kv_fwd`` on device pointers (asynchronous on ``stream``)."""
    check(lib().pa_decode_kv_fwd(ctypes.byref(desc), q_ptr, k_ptr, v_ptr, block_table_ptr,
                                 seq_lens_ptr, out_ptr, lse_ptr, workspace[0], workspace[1],
                                 stream.handle if stream is not None else None))


def decode_kv_cache(query, key_cache, value_cache, seq_lens=None, block_table=None, *,
                    scale=None, layout="hnd", kv_format=None, k_scale=1.0, v_scale=1.0,
                    max_seq_len=None, return_lse=False):
    """Decode ``query`` (batch, q_heads, head_dim) float16 over a key/value cache.

    Returns the float16 output (batch, q_heads, head_dim), and with
    ``return_lse`` also the float32 natural-log lse (batch, q_heads).
    """
    from .backend import _arena, _stream

    q = np.ascontiguousarray(query)
    if q.dtype != np.float16 or q.ndim != 3:
        raise ValueError(f"query must be float16 (batch, q_heads, head_dim), got {q.dtype} {q.shape}")
    if kv_format not in (None, "e4m3"):
        raise ValueError(f"kv_format must be None or 'e4m3', got {kv_format!r}")
    want = np.uint8 if kv_format == "e4m3" else np.float16
    k = np.ascontiguousarray(key_cache)
    v = np.ascontiguousarray(value_cache)
    if k.dtype != want or v.dtype != want:
        raise ValueError(f"caches must be {np.dtype(want).name} for kv_format={kv_format!r}")
    if k.shape != v.shape:
        raise ValueError(f"key and value caches differ in shape: {k.shape} vs {v.shape}")
    B, Hq, D = q.shape
    paged = block_table is not None
    bt = None
    if paged:
        bt = np.ascontiguousarray(block_table, dtype=np.int32)
        if bt.ndim != 2 or bt.shape[0] != B:
            raise ValueError(f"block_table must be (batch, max_pages_per_seq), got {bt.shape}")
    sl = None
    if seq_lens is not None:
        sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
        if sl.shape != (B,):
            raise ValueError(f"seq_lens must have shape ({B},), got {sl.shape}")
        if max_seq_len is None:
            max_seq_len = int(sl.max()) if B else 0
    desc = kv_cache_desc(B, Hq, D, k.shape, layout=layout, kv_format=kv_format, paged=paged,
                         max_pages_per_seq=bt.shape[1] if paged else 0, max_seq_len=max_seq_len,
                         scale=scale, k_scale=k_scale, v_scale=v_scale)
    out = np.empty((B, Hq, D), np.float16)
    lse = np.empty((B, Hq), np.float32)
    if B == 0:
        return (out, lse) if return_lse else out
    ws = kv_workspace_size(desc, paged)
    L = lib()
    st = _stream()
    arena = _arena()
    parts = [q, k, v, bt, sl]
    with arena.lock:
        ptrs = arena.carve([x.nbytes if x is not None else 0 for x in parts] +
                           [out.nbytes, lse.nbytes, ws])
        for x, p in zip(parts, ptrs):
            if x is not None:
                check(L.pa_memcpy_h2d(p, x.ctypes.data, x.nbytes, st.handle))
        dq, dk, dv, dbt, dsl, dout, dlse, dws = ptrs
        decode_kv_device(desc, dq, dk, dv, dout, block_table_ptr=dbt if paged else None,
                         seq_lens_ptr=dsl if sl is not None else None, lse_ptr=dlse, stream=st,
                         workspace=(dws, ws))
        check(L.pa_memcpy_d2h(out.ctypes.data, dout, out.nbytes, st.handle))
        check(L.pa_memcpy_d2h(lse.ctypes.data, dlse, lse.nbytes, st.handle))
        st.synchronize()
    sync_device_status()
    return (out, lse) if return_lse else out
