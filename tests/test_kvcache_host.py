"""KV-cache decode, host side: the e4m3 oracle pinned against PyTorch, the
paged-gather oracle against the dense oracle, the C struct layout, and the
plan's validation (no kernel launches)."""

from __future__ import annotations

import ctypes
import shutil
import subprocess

import numpy as np
import pytest

from oracle.kvcache import decode_kv_reference, e4m3_to_float, float_to_e4m3

from conftest import ROOT


def test_e4m3_decode_matches_torch_for_every_code():
    torch = pytest.importorskip("torch")
    codes = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).to(torch.float64).numpy()
    got = e4m3_to_float(codes)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got[~np.isnan(got)], want[~np.isnan(want)])
    assert np.nanmax(got) == 448.0 and got[1] == 2.0 ** -9


def test_e4m3_encode_matches_torch_round_to_nearest_even():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000) * s for s in (1e-3, 0.05, 1, 30, 200)])
    x = np.clip(x, -448, 448)
    pos = e4m3_to_float(np.arange(0x7F, dtype=np.uint8))
    mids = (pos[:-1] + pos[1:]) / 2            # exact ties between neighbouring codes
    x = np.concatenate([x, mids, -mids, [0.0, -0.0, 448.0, -448.0]]).astype(np.float32)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(float_to_e4m3(x), want)


def test_e4m3_encode_saturates_and_keeps_nan():
    got = float_to_e4m3(np.array([1e6, -1e6, 449.0, np.nan]))
    assert list(got) == [0x7E, 0xFE, 0x7E, 0x7F]


def page_table(B, S, page_size, rng, spare=3):
    """A shuffled block table for B sequences of up to S keys, and the page count."""
    per = -(-S // page_size)
    n_pages = B * per + spare
    return rng.permutation(n_pages)[:B * per].reshape(B, per).astype(np.int32), n_pages


def scatter_pages(x, table, n_pages, page_size, fill, layout="hnd"):
    """Scatter a dense (B, Hkv, S, D) cache into pages; unused rows hold ``fill``."""
    B, H, S, D = x.shape
    pages = np.full((n_pages, H, page_size, D), fill, dtype=x.dtype)
    for b in range(B):
        for p in range(table.shape[1]):
            rows = x[b, :, p * page_size:(p + 1) * page_size]
            pages[table[b, p], :, :rows.shape[1]] = rows
    return pages if layout == "hnd" else np.ascontiguousarray(pages.transpose(0, 2, 1, 3))


@pytest.mark.parametrize("layout", ["hnd", "nhd"])
def test_paged_oracle_equals_dense_oracle(layout):
    rng = np.random.default_rng(3)
    B, Hq, Hkv, S, D = 3, 8, 2, 70, 16
    q = rng.standard_normal((B, Hq, D))
    k = rng.standard_normal((B, Hkv, S, D))
    v = rng.standard_normal((B, Hkv, S, D))
    lens = np.array([70, 0, 33])
    table, n_pages = page_table(B, S, 16, rng)
    kp = scatter_pages(k, table, n_pages, 16, np.nan, layout)
    vp = scatter_pages(v, table, n_pages, 16, np.nan, layout)
    dense, dense_lse = decode_kv_reference(q, k, v, lens)
    paged, paged_lse = decode_kv_reference(q, kp, vp, lens, block_table=table, layout=layout)
    np.testing.assert_array_equal(dense, paged)
    np.testing.assert_array_equal(dense_lse, paged_lse)
    assert np.all(dense[1] == 0) and np.all(np.isneginf(dense_lse[1]))
    # A planted mistake in the table is visible (the comparison is not vacuous;
    # swapping two pages of one sequence would not be, attention ignores key order).
    bad = table.copy()
    bad[0, 0] = table[2, 0]
    wrong, _ = decode_kv_reference(q, kp, vp, lens, block_table=bad, layout=layout)
    assert not np.allclose(wrong[0], dense[0])


def test_fp8_oracle_dequantises_with_scales():
    rng = np.random.default_rng(4)
    q = rng.standard_normal((2, 4, 8))
    kf = rng.standard_normal((2, 1, 20, 8))
    vf = rng.standard_normal((2, 1, 20, 8))
    kq, vq = float_to_e4m3(kf / 0.5), float_to_e4m3(vf / 0.25)
    got, _ = decode_kv_reference(q, kq, vq, k_scale=0.5, v_scale=0.25, kv_format="e4m3")
    want, _ = decode_kv_reference(q, e4m3_to_float(kq) * 0.5, e4m3_to_float(vq) * 0.25)
    np.testing.assert_allclose(got, want, rtol=1e-14, atol=1e-14)


_LAYOUT_C = r"""
#include <stddef.h>
#include <stdio.h>
#include "pa_b200.h"
#define F(s, m) printf(#m " %zu\n", offsetof(s, m))
int main(void) {
  printf("size %zu\n", sizeof(pa_kv_cache_desc));
  F(pa_kv_cache_desc, q_dtype); F(pa_kv_cache_desc, kv_dtype); F(pa_kv_cache_desc, batch);
  F(pa_kv_cache_desc, q_heads); F(pa_kv_cache_desc, kv_heads); F(pa_kv_cache_desc, head_dim);
  F(pa_kv_cache_desc, max_seq_len); F(pa_kv_cache_desc, page_size); F(pa_kv_cache_desc, num_pages);
  F(pa_kv_cache_desc, max_pages_per_seq); F(pa_kv_cache_desc, key_stride);
  F(pa_kv_cache_desc, head_stride); F(pa_kv_cache_desc, page_stride); F(pa_kv_cache_desc, scale);
  F(pa_kv_cache_desc, k_scale); F(pa_kv_cache_desc, v_scale);
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_kv_cache_desc_layout_matches_the_c_compiler(tmp_path):
    from pa_b200._lib import KvCacheDesc

    src = tmp_path / "layout.c"
    src.write_text(_LAYOUT_C)
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c99", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)], check=True)
    lines = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    c = {k: int(v) for k, v in (ln.split() for ln in lines if ln)}
    assert c.pop("size") == ctypes.sizeof(KvCacheDesc)
    for name, off in c.items():
        assert getattr(KvCacheDesc, name).offset == off, name


def test_kv_cache_desc_strides():
    import pa_b200

    d = pa_b200.kv_cache_desc(4, 32, 128, (100, 8, 16, 128), layout="hnd", paged=True,
                              max_pages_per_seq=9)
    assert (d.kv_heads, d.page_size, d.num_pages, d.max_seq_len) == (8, 16, 100, 144)
    assert (d.key_stride, d.head_stride, d.page_stride) == (128, 16 * 128, 8 * 16 * 128)
    d = pa_b200.kv_cache_desc(4, 32, 128, (100, 16, 8, 128), layout="nhd", paged=True,
                              max_pages_per_seq=9, kv_format="e4m3")
    assert (d.kv_heads, d.page_size) == (8, 16)
    assert (d.key_stride, d.head_stride, d.page_stride) == (8 * 128, 128, 16 * 8 * 128)
    assert d.kv_dtype == 6 and d.q_dtype == 1
    with pytest.raises(ValueError, match="multiple of kv_heads"):
        pa_b200.kv_cache_desc(4, 30, 128, (100, 8, 16, 128))


@pytest.mark.parametrize("change,status,msg", [
    (dict(page_size=12), 2, "multiple of 8"),
    (dict(max_pages_per_seq=3), 1, "cover max_seq_len"),
    (dict(head_dim=96), 2, "64 or 128"),
    (dict(q_heads=68), 2, "at most 16"),
    (dict(kv_dtype=2), 2, "query's dtype or fp8"),
    (dict(scale=float("nan")), 1, "finite"),
])
def test_plan_rejects_bad_descriptors(change, status, msg):
    import pa_b200
    from pa_b200._lib import PaError, check, lib

    d = pa_b200.kv_cache_desc(2, 16, 128, (64, 4, 16, 128), paged=True, max_pages_per_seq=8)
    for k, v in change.items():
        setattr(d, k, v)
    n = ctypes.c_size_t(0)
    with pytest.raises(PaError, match=msg) as err:
        check(lib().pa_decode_kv_workspace_size(ctypes.byref(d), 1, ctypes.byref(n)))
    assert err.value.status == status


def test_workspace_size_counts_split_partials():
    import pa_b200
    from pa_b200._lib import check, lib

    d = pa_b200.kv_cache_desc(2, 16, 128, (64, 4, 16, 128), paged=True, max_pages_per_seq=8)
    n = ctypes.c_size_t(0)
    check(lib().pa_decode_kv_workspace_size(ctypes.byref(d), 1, ctypes.byref(n)))
    assert n.value > 0 and n.value % (2 * 16 * (128 + 2) * 4) == 0


def _kv_args():
    rng = np.random.default_rng(5)
    q = rng.standard_normal((2, 8, 64)).astype(np.float16)
    k = rng.standard_normal((2, 2, 32, 64)).astype(np.float16)
    return q, k, k.copy()


@pytest.mark.parametrize("change,msg", [
    (lambda q, k, v: (q.astype(np.float32), k, v, {}), "query must be float16"),
    (lambda q, k, v: (q[0], k, v, {}), "query must be float16"),
    (lambda q, k, v: (q, k, v, {"kv_format": "e5m2"}), "kv_format must be"),
    (lambda q, k, v: (q, k.astype(np.float32), v, {}), "caches must be float16"),
    (lambda q, k, v: (q, k, v, {"kv_format": "e4m3"}), "caches must be uint8"),
    (lambda q, k, v: (q, k, v[:, :, :16], {}), "differ in shape"),
    (lambda q, k, v: (q, k, v, {"block_table": np.zeros((3, 2), np.int32)}), "block_table must be"),
    (lambda q, k, v: (q, k, v, {"seq_lens": np.array([1, 2, 3])}), "seq_lens must have shape"),
    (lambda q, k, v: (q, k, v, {"layout": "bhsd"}), "layout must be one of"),
    (lambda q, k, v: (q[:, :, :32], k, v, {}), "does not match the query's"),
    (lambda q, k, v: (q[:, :7], k, v, {}), "multiple of kv_heads"),
])
def test_decode_kv_cache_rejects_bad_arguments_before_any_device_work(change, msg):
    """Argument errors are raised by the host layer, before the library is touched."""
    import pa_b200

    q, k, v, kw = change(*_kv_args())
    with pytest.raises(ValueError, match=msg):
        pa_b200.decode_kv_cache(q, k, v, **kw)
