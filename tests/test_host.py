"""Host-side logic of the CUDA backend that needs no GPU.

Covers the descriptor planning (broadcast leading dims, zero strides, the
grouped-query index division), argument validation against the reference's
own messages, registration through a registry callable, and that
``libpa_b200.so`` loads and exports every function ``include/pa_b200.h``
declares (no compute call is made here).
"""

from __future__ import annotations

import ctypes
import json
import re

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
import pa_b200
from pa_b200 import _lib, plan_call
from pa_b200.plan import compute_dtype
from pa_b200.validation import validate


def _desc_tuple(arr, n):
    return [arr[i] for i in range(n)]


def test_plan_dense_bhsd_gqa():
    p = plan_call((2, 8, 5, 16), (2, 2, 7, 16), (2, 2, 7, 4), np.float32, np.float32, np.float32,
                  group=4)
    d = p.desc
    assert p.out_shape == (2, 8, 5, 4)
    assert d.nlead == 2 and _desc_tuple(d.lead, 2) == [2, 8]
    assert _desc_tuple(d.q_lead_stride, 2) == [8 * 5 * 16, 5 * 16]
    assert _desc_tuple(d.k_lead_stride, 2) == [2 * 7 * 16, 7 * 16]
    assert _desc_tuple(d.v_lead_stride, 2) == [2 * 7 * 4, 7 * 4]
    assert d.gqa_axis == 1 and d.gqa_group == 4
    assert d.scale == pytest.approx(1 / 4)


def test_plan_broadcast_mask_and_operands():
    # q has no batch axis; the mask brings one (reference broadcasting via np.matmul / np.where).
    p = plan_call((5, 8), (3, 7, 8), (3, 7, 4), np.float64, np.float64, np.float64,
                  mask_shape=(1, 5, 7), mask_dtype=np.bool_)
    d = p.desc
    assert p.out_shape == (3, 5, 4)
    assert _desc_tuple(d.q_lead_stride, 1) == [0]
    assert _desc_tuple(d.k_lead_stride, 1) == [56]
    assert _desc_tuple(d.m_lead_stride, 1) == [0]
    assert d.m_row_stride == 7 and d.m_col_stride == 1
    assert d.mask_kind == _lib.PA_MASK_BOOL and d.mask_dtype == _lib.PA_BOOL


def test_plan_mask_row_and_column_broadcast():
    p = plan_call((2, 5, 8), (2, 7, 8), (2, 7, 4), np.float32, np.float32, np.float32,
                  mask_shape=(7,), mask_dtype=np.float32)
    d = p.desc
    assert p.mask_shape == (1, 7)
    assert d.m_row_stride == 0 and d.m_col_stride == 1
    assert d.mask_kind == _lib.PA_MASK_ADD and d.mask_dtype == _lib.PA_F32
    with pytest.raises(ValueError, match="broadcastable"):
        plan_call((2, 5, 8), (2, 7, 8), (2, 7, 4), np.float32, np.float32, np.float32,
                  mask_shape=(4, 7), mask_dtype=np.bool_)


def test_plan_causal_ignores_no_mask_and_sets_flag():
    p = plan_call((1, 4, 6, 8), (1, 4, 6, 8), (1, 4, 6, 4), np.float16, np.float16, np.float16,
                  is_causal=True, scale=0.5)
    assert p.desc.is_causal == 1 and p.desc.scale == 0.5 and p.cdt == np.float16


@pytest.mark.parametrize("dts,mask,want", [
    ((np.float16,) * 3, None, np.float16),
    ((np.float16,) * 3, np.bool_, np.float16),
    ((np.float16,) * 3, np.float32, np.float16),
    ((np.float16,) * 3, np.float64, np.float64),
    ((np.float32,) * 3, None, np.float32),
    ((np.float32, np.float64, np.float64), None, np.float64),
    ((np.float32,) * 3, np.float64, np.float64),
    ((np.float16, np.float32, np.float16), None, np.float32),
    ((np.int64,) * 3, None, np.float64),
])
def test_compute_dtype(dts, mask, want):
    assert compute_dtype(*dts, mask) == np.dtype(want)


def test_validation_messages_match_reference():
    golden = json.loads((GOLDEN / "messages.json").read_text())
    z = np.zeros
    calls = {
        "ndim": ((z(4), z((3, 4)), z((3, 4))), {}),
        "embed": ((z((5, 8)), z((6, 7)), z((6, 3))), {}),
        "seq": ((z((5, 8)), z((6, 8)), z((7, 3))), {}),
        "causal+mask": ((z((4, 4, 8)), z((4, 4, 8)), z((4, 4, 8))),
                        {"attn_mask": np.ones((4, 4), bool), "is_causal": True}),
        "gqa-ndim": ((z((5, 8)), z((7, 8)), z((7, 4))), {"enable_gqa": True}),
        "gqa-multiple": ((z((2, 8, 5, 8)), z((2, 3, 7, 8)), z((2, 3, 7, 4))), {"enable_gqa": True}),
        "gqa-kv-heads": ((z((2, 8, 5, 8)), z((2, 2, 7, 8)), z((2, 4, 7, 4))), {"enable_gqa": True}),
        "gqa-zero": ((z((2, 0, 5, 8)), z((2, 2, 7, 8)), z((2, 2, 7, 4))), {"enable_gqa": True}),
    }
    for key, (args, kw) in calls.items():
        q, k, v = args
        with pytest.raises(Exception) as info:
            validate(q, k, v, kw.get("attn_mask"), kw.get("dropout_p", 0.0),
                     kw.get("is_causal", False), kw.get("enable_gqa", False))
        assert [type(info.value).__name__, str(info.value)] == golden[f"{key}|reference"], key
    with pytest.raises(NotImplementedError, match="dropout_p"):
        validate(z((2, 4, 8)), z((2, 4, 8)), z((2, 4, 8)), None, 0.1, False, False)


def test_register_uses_the_given_registry(monkeypatch):
    seen = {}

    def registry(name, backend, *, overwrite=False):
        seen[name] = (backend, overwrite)

    monkeypatch.setattr(pa_b200, "available", lambda: True)
    assert pa_b200.register(registry=registry, overwrite=True)
    assert seen == {"cuda": (pa_b200.scaled_dot_product_attention, True)}


def test_register_is_a_noop_without_a_gpu(monkeypatch):
    monkeypatch.setattr(pa_b200, "available", lambda: False)
    calls = []
    assert not pa_b200.register(registry=lambda *a, **k: calls.append(a))
    assert calls == []


def test_register_into_the_real_registry_when_present(monkeypatch, reference_package):
    pa = reference_package
    from portable_attention.dispatch import _REGISTRY

    saved = dict(_REGISTRY)
    monkeypatch.setattr(pa_b200, "available", lambda: True)
    try:
        assert pa_b200.register()
        assert pa.get_backend("cuda") is pa_b200.scaled_dot_product_attention
        assert isinstance(pa.get_backend("cuda"), pa.SdpaBackend)
        # auto dispatch is untouched (dispatch.py:146-159)
        assert pa.dispatch._auto_select(np.zeros((2, 3, 5, 8))) is pa.get_backend("fused")
    finally:
        _REGISTRY.clear()
        _REGISTRY.update(saved)


def _header_functions():
    text = (ROOT / "include" / "pa_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(pa_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_header_function():
    names = _header_functions()
    assert "pa_sdpa_fwd" in names and "pa_ring_fwd" in names
    h = _lib.lib()
    for name in names:
        assert hasattr(h, name), name
    assert set(names) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"
    assert h.pa_version() >= 100


def test_sdpa_desc_layout_matches_header():
    # int32 dtype, nlead; 5 x 6 int64 arrays; 7 int64; 4 int32; 2 int64; 2 int32; double
    assert ctypes.sizeof(_lib.SdpaDesc) == 8 + 5 * 6 * 8 + 7 * 8 + 4 * 4 + 2 * 8 + 2 * 4 + 8


def test_missing_library_raises_not_falls_back(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_handle", None)
    monkeypatch.setenv("PA_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(_lib.LibraryError):
        _lib.lib()
    assert not pa_b200.available()


def test_decode_null_operands_rejected_before_any_launch():
    """NULL q/k/v/out fail with PA_ERR_INVALID on the host (both decode entry points)."""
    plan = pa_b200.plan_call((2, 8, 1, 128), (2, 2, 64, 128), (2, 2, 64, 128),
                             np.float16, np.float16, np.float16, group=4)
    h = _lib.lib()
    rc = h.pa_decode_fwd(ctypes.byref(plan.desc), None, None, None, None, None, None, 0, None)
    assert rc == _lib.PA_ERR_INVALID
    assert "null" in h.pa_last_error().decode()
    rc = h.pa_decode_fwd_static(ctypes.byref(plan.desc), None, None, None, None, None, None, None)
    assert rc == _lib.PA_ERR_INVALID
    assert "null" in h.pa_last_error().decode()


def test_ordinary_numpy_memory_is_not_reported_pinned():
    from pa_b200.device import is_pinned

    assert not is_pinned(np.zeros(1024, np.float32))


def test_wait_selftest_rejects_out_of_range_limits():
    h = _lib.lib()
    for bad in (0, -5, 1000001):
        assert h.pa_selftest_wait_timeout(bad, None) == _lib.PA_ERR_INVALID


def test_backward_argument_errors_on_the_host():
    """sdpa_backward's scope checks run before any device work (no GPU needed)."""
    import pa_b200

    z = np.zeros((1, 2, 8, 64), np.float16)
    with pytest.raises(NotImplementedError, match="head dim 64 or 128"):
        pa_b200.sdpa_backward(z[..., :32], z[..., :32], z[..., :32], z[..., :32])
    with pytest.raises(NotImplementedError, match="float16"):
        pa_b200.sdpa_backward(*(z.astype(np.float32),) * 4)
    with pytest.raises(NotImplementedError, match="attn_mask"):
        pa_b200.sdpa_backward(z, z, z, z, attn_mask=np.ones((8, 8), bool))
    with pytest.raises(NotImplementedError, match="dropout_p"):
        pa_b200.sdpa_backward(z, z, z, z, dropout_p=0.1)
    with pytest.raises(NotImplementedError, match="head axis"):
        pa_b200.sdpa_backward(z[0, 0], z[0, 0], z[0, 0], z[0, 0])
    with pytest.raises(ValueError, match="dout shape"):
        pa_b200.sdpa_backward(z, z, z, z[..., :4, :])
    with pytest.raises(ValueError):
        pa_b200.sdpa_backward(z, z[..., :32], z, z)  # E mismatch: the reference's validation message
