"""KV-cache decode parity on the GPU: varlen, paged (hnd / nhd, page sizes 8
to 64) and fp8 e4m3 caches, against the float64 oracle of oracle/kvcache.py.

Rows of the caches past each sequence's length (and spare pages) are filled
with NaN, so a kernel that touched them would fail loudly. Tolerances:
fp16 output 2e-3 abs / 2e-3 rel; bf16 output 1.6e-2 abs / 1e-2 rel (8
significand bits); lse 2e-3 abs / 1e-4 rel. fp8 inputs are exact e4m3
values, so the oracle sees exactly what the kernel sees.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle.kvcache import decode_kv_reference, e4m3_to_float, float_to_e4m3

pytestmark = pytest.mark.gpu


def page_table(B, S, page_size, rng, spare=3):
    per = -(-S // page_size)
    n_pages = B * per + spare
    return rng.permutation(n_pages)[:B * per].reshape(B, per).astype(np.int32), n_pages


def scatter_pages(x, table, n_pages, page_size, fill, layout="hnd"):
    B, H, S, D = x.shape
    pages = np.full((n_pages, H, page_size, D), fill, dtype=x.dtype)
    for b in range(B):
        for p in range(table.shape[1]):
            rows = x[b, :, p * page_size:(p + 1) * page_size]
            pages[table[b, p], :, :rows.shape[1]] = rows
    return pages if layout == "hnd" else np.ascontiguousarray(pages.transpose(0, 2, 1, 3))


def blank_tails(x, lens, fill):
    """Overwrite rows past each sequence's length of a dense (B, H, S, D) cache."""
    x = x.copy()
    for b, n in enumerate(lens):
        x[b, :, n:] = fill
    return x


def check(got, got_lse, want, want_lse, atol=2e-3, rtol=2e-3):
    assert np.isfinite(got.astype(np.float64)).all()
    np.testing.assert_allclose(got.astype(np.float64), want, rtol=rtol, atol=atol)
    np.testing.assert_allclose(got_lse, want_lse, rtol=1e-4, atol=2e-3)


@pytest.mark.parametrize("D,hq,hkv", [(128, 16, 4), (64, 8, 1), (128, 8, 8)])
def test_varlen_contiguous_cache(D, hq, hkv):
    import pa_b200

    rng = np.random.default_rng(D + hq)
    B, S = 5, 3000
    lens = np.array([3000, 0, 1, 777, 2049], dtype=np.int32)
    q = rng.standard_normal((B, hq, D)).astype(np.float16)
    k = blank_tails(rng.standard_normal((B, hkv, S, D)).astype(np.float16), lens, np.nan)
    v = blank_tails(rng.standard_normal((B, hkv, S, D)).astype(np.float16), lens, np.nan)
    out, lse = pa_b200.decode_kv_cache(q, k, v, lens, return_lse=True)
    want, want_lse = decode_kv_reference(q, k, v, lens)
    check(out, lse, want, want_lse)
    assert np.all(out[1] == 0) and np.all(np.isneginf(lse[1]))


@pytest.mark.parametrize("page_size,layout,D,hq,hkv", [
    (16, "hnd", 64, 16, 2), (32, "nhd", 128, 4, 4), (8, "hnd", 128, 8, 4), (64, "nhd", 64, 8, 1),
    (16, "nhd", 128, 32, 8), (16, "hnd", 128, 32, 2), (32, "hnd", 64, 12, 1),
])
def test_paged_cache(page_size, layout, D, hq, hkv):
    import pa_b200

    rng = np.random.default_rng(page_size * 7 + D)
    B, S = 4, 1500
    lens = np.array([1500, 0, 17, 1023], dtype=np.int32)
    q = rng.standard_normal((B, hq, D)).astype(np.float16)
    k = rng.standard_normal((B, hkv, S, D)).astype(np.float16)
    v = rng.standard_normal((B, hkv, S, D)).astype(np.float16)
    table, n_pages = page_table(B, S, page_size, rng)
    kp = scatter_pages(blank_tails(k, lens, np.nan), table, n_pages, page_size, np.nan, layout)
    vp = scatter_pages(blank_tails(v, lens, np.nan), table, n_pages, page_size, np.nan, layout)
    out, lse = pa_b200.decode_kv_cache(q, kp, vp, lens, table, layout=layout, return_lse=True)
    want, want_lse = decode_kv_reference(q, k, v, lens)
    check(out, lse, want, want_lse)


@pytest.mark.parametrize("paged,D,hq,hkv", [(True, 128, 32, 8), (False, 64, 16, 2), (True, 64, 8, 8),
                                             (True, 128, 24, 2), (False, 128, 14, 1)])
def test_fp8_e4m3_cache(paged, D, hq, hkv):
    import pa_b200

    rng = np.random.default_rng(40 + D + hq)
    B, S = 3, 2500
    lens = np.array([2500, 1, 1290], dtype=np.int32)
    k_scale, v_scale = 0.02, 0.05
    q = rng.standard_normal((B, hq, D)).astype(np.float16)
    kq = blank_tails(float_to_e4m3(rng.standard_normal((B, hkv, S, D)) / k_scale), lens, 0x7F)
    vq = blank_tails(float_to_e4m3(rng.standard_normal((B, hkv, S, D)) / v_scale), lens, 0x7F)
    kw = dict(kv_format="e4m3", k_scale=k_scale, v_scale=v_scale, return_lse=True)
    if paged:
        table, n_pages = page_table(B, S, 16, rng)
        out, lse = pa_b200.decode_kv_cache(q, scatter_pages(kq, table, n_pages, 16, 0x7F),
                                           scatter_pages(vq, table, n_pages, 16, 0x7F), lens, table, **kw)
    else:
        out, lse = pa_b200.decode_kv_cache(q, kq, vq, lens, **kw)
    want, want_lse = decode_kv_reference(q, kq, vq, lens, k_scale=k_scale, v_scale=v_scale,
                                         kv_format="e4m3")
    check(out, lse, want, want_lse)


def to_bf16_bits(x):
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def from_bf16_bits(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("fp8", [True, False])
def test_bf16_query_through_the_c_abi(fp8):
    import pa_b200
    from pa_b200._lib import check as ok, lib
    from pa_b200.device import DeviceBuffer, Stream

    rng = np.random.default_rng(77 + fp8)
    B, hq, hkv, D, S, ps = 3, 16, 4, 128, 900, 32
    lens = np.array([900, 500, 33], dtype=np.int32)
    qb = to_bf16_bits(rng.standard_normal((B, hq, D)))
    if fp8:
        k = float_to_e4m3(rng.standard_normal((B, hkv, S, D)) * 4)
        v = float_to_e4m3(rng.standard_normal((B, hkv, S, D)) * 4)
        fill = 0x7F
    else:
        k = to_bf16_bits(rng.standard_normal((B, hkv, S, D)))
        v = to_bf16_bits(rng.standard_normal((B, hkv, S, D)))
        fill = 0x7FC0  # bf16 NaN
    table, n_pages = page_table(B, S, ps, rng)
    kp = scatter_pages(blank_tails(k, lens, fill), table, n_pages, ps, fill)
    vp = scatter_pages(blank_tails(v, lens, fill), table, n_pages, ps, fill)
    desc = pa_b200.kv_cache_desc(B, hq, D, kp.shape, q_dtype="bf16", kv_format="e4m3" if fp8 else None,
                                 paged=True, max_pages_per_seq=table.shape[1], max_seq_len=S,
                                 k_scale=0.25 if fp8 else 1.0, v_scale=0.25 if fp8 else 1.0)
    st = Stream()
    bufs = []
    for x in (qb, kp, vp, table, lens):
        buf = DeviceBuffer(x.nbytes)
        ok(lib().pa_memcpy_h2d(buf.ptr, x.ctypes.data, x.nbytes, st.handle))
        bufs.append(buf)
    out, lse = DeviceBuffer(qb.nbytes), DeviceBuffer(B * hq * 4)
    pa_b200.decode_kv_device(desc, bufs[0].ptr, bufs[1].ptr, bufs[2].ptr, out.ptr,
                             block_table_ptr=bufs[3].ptr, seq_lens_ptr=bufs[4].ptr, lse_ptr=lse.ptr,
                             stream=st)
    got = np.empty_like(qb)
    got_lse = np.empty((B, hq), np.float32)
    ok(lib().pa_memcpy_d2h(got.ctypes.data, out.ptr, got.nbytes, st.handle))
    ok(lib().pa_memcpy_d2h(got_lse.ctypes.data, lse.ptr, got_lse.nbytes, st.handle))
    st.synchronize()
    pa_b200.sync_device_status()
    q = from_bf16_bits(qb)
    if fp8:
        want, want_lse = decode_kv_reference(q, k, v, lens, k_scale=0.25, v_scale=0.25, kv_format="e4m3")
    else:
        want, want_lse = decode_kv_reference(q, from_bf16_bits(k), from_bf16_bits(v), lens)
    check(from_bf16_bits(got), got_lse, want, want_lse, atol=1.6e-2, rtol=1e-2)


def test_bad_block_table_entry_and_length_are_reported():
    import pa_b200
    from pa_b200._lib import PaError

    rng = np.random.default_rng(9)
    B, hq, hkv, D, S, ps = 2, 8, 2, 128, 256, 16
    q = rng.standard_normal((B, hq, D)).astype(np.float16)
    k = rng.standard_normal((B, hkv, S, D)).astype(np.float16)
    table, n_pages = page_table(B, S, ps, rng)
    kp = scatter_pages(k, table, n_pages, ps, 0.0)
    bad = table.copy()
    bad[1, 3] = n_pages + 1000
    with pytest.raises(PaError, match="block-table entry") as err:
        pa_b200.decode_kv_cache(q, kp, kp, np.array([S, S], np.int32), bad)
    assert err.value.status == 1
    # The device recovered: the same call with a good table works.
    out = pa_b200.decode_kv_cache(q, kp, kp, np.array([S, S], np.int32), table)
    assert np.isfinite(out.astype(np.float32)).all()
    with pytest.raises(PaError, match="sequence length") as err:
        pa_b200.decode_kv_cache(q, kp, kp, np.array([S, 5], np.int32), table, max_seq_len=100)
    assert err.value.status == 1


def test_dense_decode_unchanged_through_both_entry_points():
    """pa_decode_fwd (dense operands) and pa_decode_kv_fwd (one page per sequence) agree exactly."""
    import pa_b200

    rng = np.random.default_rng(12)
    q = rng.standard_normal((4, 16, 1, 128)).astype(np.float16)
    k = rng.standard_normal((4, 4, 5000, 128)).astype(np.float16)
    v = rng.standard_normal((4, 4, 5000, 128)).astype(np.float16)
    dense = pa_b200.scaled_dot_product_attention(q, k, v, enable_gqa=True)[:, :, 0]
    cached = pa_b200.decode_kv_cache(q[:, :, 0], k, v)
    np.testing.assert_array_equal(dense, cached)
