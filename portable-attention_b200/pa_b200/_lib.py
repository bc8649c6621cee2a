"""ctypes binding of ``libpa_b200.so`` (declared in ``include/pa_b200.h``).

The library is looked up in ``$PA_B200_LIB`` or next to this file. There is no
fallback: if it cannot be loaded, :func:`lib` raises :class:`LibraryError`, so a
caller can never silently get a CPU result from this backend.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

__all__ = [
    "PA_BF16", "PA_BOOL", "PA_F16", "PA_F32", "PA_F64", "PA_FP8_E4M3", "PA_MASK_ADD",
    "PA_MASK_BOOL", "PA_MASK_NONE", "PA_MAX_LEAD", "KvCacheDesc", "LibraryError", "PaError",
    "SdpaDesc", "check", "lib", "library_path",
]

PA_OK, PA_ERR_INVALID, PA_ERR_UNSUPPORTED, PA_ERR_CUDA, PA_ERR_TIMEOUT, PA_ERR_NCCL, PA_ERR_NOMEM = range(7)
PA_F16, PA_BF16, PA_F32, PA_F64, PA_BOOL, PA_FP8_E4M3 = 1, 2, 3, 4, 5, 6
PA_MASK_NONE, PA_MASK_BOOL, PA_MASK_ADD = 0, 1, 2
PA_MAX_LEAD = 6

_STATUS_NAMES = {
    PA_ERR_INVALID: "invalid argument",
    PA_ERR_UNSUPPORTED: "unsupported",
    PA_ERR_CUDA: "CUDA error",
    PA_ERR_TIMEOUT: "device wait timed out",
    PA_ERR_NCCL: "NCCL error",
    PA_ERR_NOMEM: "out of memory",
}


class LibraryError(RuntimeError):
    """``libpa_b200.so`` is missing or cannot be loaded."""


class PaError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{_STATUS_NAMES.get(status, 'error')} ({status}): {message}")
        self.status = status


class SdpaDesc(ctypes.Structure):
    """Mirror of ``pa_sdpa_desc`` (include/pa_b200.h)."""

    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("nlead", ctypes.c_int32),
        ("lead", ctypes.c_int64 * PA_MAX_LEAD),
        ("q_lead_stride", ctypes.c_int64 * PA_MAX_LEAD),
        ("k_lead_stride", ctypes.c_int64 * PA_MAX_LEAD),
        ("v_lead_stride", ctypes.c_int64 * PA_MAX_LEAD),
        ("m_lead_stride", ctypes.c_int64 * PA_MAX_LEAD),
        ("L", ctypes.c_int64),
        ("S", ctypes.c_int64),
        ("E", ctypes.c_int64),
        ("Ev", ctypes.c_int64),
        ("q_row_stride", ctypes.c_int64),
        ("k_row_stride", ctypes.c_int64),
        ("v_row_stride", ctypes.c_int64),
        ("gqa_axis", ctypes.c_int32),
        ("gqa_group", ctypes.c_int32),
        ("mask_kind", ctypes.c_int32),
        ("mask_dtype", ctypes.c_int32),
        ("m_row_stride", ctypes.c_int64),
        ("m_col_stride", ctypes.c_int64),
        ("is_causal", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("scale", ctypes.c_double),
    ]


class KvCacheDesc(ctypes.Structure):
    """Mirror of ``pa_kv_cache_desc`` (include/pa_b200.h)."""

    _fields_ = [
        ("q_dtype", ctypes.c_int32),
        ("kv_dtype", ctypes.c_int32),
        ("batch", ctypes.c_int64),
        ("q_heads", ctypes.c_int64),
        ("kv_heads", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("max_seq_len", ctypes.c_int64),
        ("page_size", ctypes.c_int64),
        ("num_pages", ctypes.c_int64),
        ("max_pages_per_seq", ctypes.c_int64),
        ("key_stride", ctypes.c_int64),
        ("head_stride", ctypes.c_int64),
        ("page_stride", ctypes.c_int64),
        ("scale", ctypes.c_double),
        ("k_scale", ctypes.c_float),
        ("v_scale", ctypes.c_float),
    ]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_DESC = ctypes.POINTER(SdpaDesc)
_F32P = ctypes.POINTER(ctypes.c_float)

# name -> argtypes; every symbol returns pa_status (int32) unless listed in _RESTYPES.
SIGNATURES = {
    "pa_version": [],
    "pa_last_error": [],
    "pa_init": [ctypes.POINTER(_I32)],
    "pa_set_device": [_I32],
    "pa_get_device": [ctypes.POINTER(_I32)],
    "pa_device_status": [ctypes.POINTER(_I32)],
    "pa_selftest_wait_timeout": [_I32, _P],
    "pa_malloc": [ctypes.POINTER(_P), ctypes.c_size_t],
    "pa_free": [_P],
    "pa_host_alloc": [ctypes.POINTER(_P), ctypes.c_size_t],
    "pa_host_free": [_P],
    "pa_memcpy_h2d": [_P, _P, ctypes.c_size_t, _P],
    "pa_memcpy_d2h": [_P, _P, ctypes.c_size_t, _P],
    "pa_memcpy_d2d": [_P, _P, ctypes.c_size_t, _P],
    "pa_memset": [_P, _I32, ctypes.c_size_t, _P],
    "pa_stream_create": [ctypes.POINTER(_P)],
    "pa_stream_destroy": [_P],
    "pa_stream_sync": [_P],
    "pa_event_create": [ctypes.POINTER(_P)],
    "pa_event_destroy": [_P],
    "pa_event_record": [_P, _P],
    "pa_event_sync": [_P],
    "pa_host_is_pinned": [_P, ctypes.POINTER(_I32)],
    "pa_stream_wait_event": [_P, _P],
    "pa_event_elapsed_ms": [_P, _P, ctypes.POINTER(ctypes.c_float)],
    "pa_sdpa_fwd": [_DESC, _P, _P, _P, _P, _P, _P, _P],
    "pa_decode_workspace_size": [_DESC, ctypes.POINTER(ctypes.c_size_t)],
    "pa_decode_fwd": [_DESC, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    "pa_decode_fwd_static": [_DESC, _P, _P, _P, _P, _P, _P, _P],
    "pa_decode_kv_workspace_size": [ctypes.POINTER(KvCacheDesc), _I32, ctypes.POINTER(ctypes.c_size_t)],
    "pa_decode_kv_fwd": [ctypes.POINTER(KvCacheDesc), _P, _P, _P, _P, _P, _P, _P, _P, ctypes.c_size_t, _P],
    "pa_fwd_tile_plan": [_I32, _I32, _P],
    "pa_shard_fwd": [_I32, _P, _DESC, _P, _P, _P, _P, _P, _P],
    "pa_sdpa_bwd": [_DESC, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
    "pa_comm_unique_id": [ctypes.c_char_p],
    "pa_comm_init": [ctypes.POINTER(_P), ctypes.c_char_p, _I32, _I32],
    "pa_comm_destroy": [_P],
    "pa_comm_wait": [_P, _P, _I32],
    "pa_comm_profile_start": [_P],
    "pa_comm_profile_read": [_P, _P],
    "pa_ring_fwd": [_P, _DESC, _P, _P, _P, _P, _P, _P],
    "pa_ring_bwd": [_P, _DESC, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P],
}
_RESTYPES = {"pa_version": _I32, "pa_last_error": ctypes.c_char_p}

_lock = threading.Lock()
_handle: ctypes.CDLL | None = None


def library_path() -> Path:
    env = os.environ.get("PA_B200_LIB")
    return Path(env) if env else Path(__file__).resolve().parent / "libpa_b200.so"


def _prefer_python_nccl() -> None:
    """Point the library's lazy NCCL load at the pip ``nvidia-nccl`` build when present.

    Frameworks in the same process (PyTorch) load that build; using the same
    file avoids two different ``libnccl.so.2`` in one process.
    """
    if os.environ.get("PA_B200_NCCL"):
        return
    try:
        import importlib.util

        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return
    for base in (spec.submodule_search_locations or []) if spec else []:
        cand = Path(base) / "lib" / "libnccl.so.2"
        if cand.exists():
            os.environ["PA_B200_NCCL"] = str(cand)
            return


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library, with every signature declared."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            path = library_path()
            if not path.exists():
                raise LibraryError(
                    f"libpa_b200.so not found at {path}; build it with "
                    "`python portable-attention_b200/build.py`")
            _prefer_python_nccl()
            try:
                h = ctypes.CDLL(str(path))
            except OSError as exc:
                raise LibraryError(f"cannot load {path}: {exc}") from exc
            for name, argtypes in SIGNATURES.items():
                fn = getattr(h, name)
                fn.argtypes = argtypes
                fn.restype = _RESTYPES.get(name, _I32)
            _handle = h
    return _handle


def check(status: int) -> None:
    """Raise :class:`PaError` with the library's message for a non-zero status."""
    if status != PA_OK:
        msg = lib().pa_last_error() or b""
        raise PaError(status, msg.decode(errors="replace"))
