"""pa_b200 -- a B200 (sm_100a) CUDA backend for portable-attention.

The backend plugs into the reference project's own seam: it is one more
``SdpaBackend`` callable (``src/portable_attention/dispatch.py:53-76``) that
:func:`register` adds with ``portable_attention.register_backend``
(``dispatch.py:92-120``). Nothing else in the reference changes: ``auto``
dispatch, ``__all__`` and the conformance kit stay as they are, and a host
without a GPU simply never registers ``cuda``.

    import portable_attention as pa
    import pa_b200

    pa_b200.register()                     # adds "cuda" when a GPU is present
    out = pa.get_backend("cuda")(q, k, v, is_causal=True)
"""

from __future__ import annotations

from ._lib import LibraryError, PaError, library_path
from .autograd import forward_with_lse, sdpa_backward
from .backend import scaled_dot_product_attention, sdpa_device, sdpa_sharded
from .kvcache import decode_kv_cache, decode_kv_device, kv_cache_desc
from .device import (DeviceBuffer, Event, Stream, current_device, device_count, pinned_empty,
                     set_device, sync_device_status)
from .plan import compute_dtype, plan_call
from .tiling import B200_LIMITS, plan_tcgen05_tiles

__all__ = [
    "B200_LIMITS", "DeviceBuffer", "Event", "LibraryError", "PaError", "Stream", "available", "compute_dtype",
    "current_device", "decode_kv_cache", "decode_kv_device", "device_count", "forward_with_lse",
    "kv_cache_desc", "library_path", "plan_tcgen05_tiles", "pinned_empty",
    "plan_call", "register", "scaled_dot_product_attention", "sdpa_backward", "sdpa_device", "sdpa_sharded",
    "set_device", "sync_device_status",
]

__version__ = "0.1.0"


def available() -> bool:
    """True when the native library loads and at least one CUDA device is visible."""
    try:
        return device_count() > 0
    except LibraryError:
        return False


def register(name: str = "cuda", *, overwrite: bool = False, registry=None) -> bool:
    """Register the backend under ``name`` if a GPU is usable; return whether it did.

    ``registry`` defaults to ``portable_attention.register_backend``; any
    callable with that signature (name, backend, *, overwrite) works, which is
    how the tests exercise registration without the reference installed.
    """
    if registry is None:
        import portable_attention

        registry = portable_attention.register_backend
    if not available():
        return False
    registry(name, scaled_dot_product_attention, overwrite=overwrite)
    return True
