"""NumPy restatement of decode over a key/value cache (oracle; test infrastructure).

The reference's SdpaBackend takes dense key/value tensors
(``src/portable_attention/dispatch.py:53-76``). A serving stack keeps keys and
values in a cache instead: per-sequence lengths, optionally split into pages
named by a block table, optionally stored as fp8. Decoding from such a cache
is defined here as exactly the reference's algorithm on the gathered,
dequantised keys of each sequence:

* gather keys ``[0, seq_lens[b])`` of sequence ``b`` (key ``j`` is row
  ``j % page_size`` of page ``block_table[b, j // page_size]``, or row ``j``
  of page ``b`` without a table);
* dequantise: ``k * k_scale``, ``v * v_scale`` (per-tensor scales, applied to
  the decoded fp8 values);
* ``reference_sdpa`` (``reference.py:56-163``) with the length-1 query and
  ``enable_gqa``; the lse is ``reference_lse`` (natural log);
* a sequence of length 0 has no keys: its output row is zero and its lse
  ``-inf`` (the convention the library's fully-masked rows follow,
  ``reference.py:151-160``).

The fp8 format is OCP FP8 E4M3 ("e4m3fn": sign, 4 exponent bits with bias 7,
3 mantissa bits, subnormals, no infinities, ``0x7f``/``0xff`` NaN, largest
finite 448). :func:`e4m3_to_float` decodes from that definition and
:func:`float_to_e4m3` rounds to nearest-even with saturation at +-448 (how
fp8 KV caches are written). Both are pinned against PyTorch's
``torch.float8_e4m3fn`` by the CPU tests.
"""

from __future__ import annotations

import numpy as np

from .sdpa import reference_lse, reference_sdpa

__all__ = ["decode_kv_reference", "e4m3_to_float", "float_to_e4m3", "gather_sequence"]

E4M3_MAX = 448.0


def _e4m3_table() -> np.ndarray:
    codes = np.arange(256)
    sign = np.where(codes & 0x80, -1.0, 1.0)
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    normal = np.ldexp(1.0 + man / 8.0, exp - 7)
    subnormal = np.ldexp(man / 8.0, -6)
    vals = sign * np.where(exp > 0, normal, subnormal)
    vals[(codes & 0x7F) == 0x7F] = np.nan
    return vals


_TABLE = _e4m3_table()
_POSITIVE = _TABLE[:0x7F]          # codes 0x00..0x7e, increasing


def e4m3_to_float(bits) -> np.ndarray:
    """Decode e4m3 bit patterns (uint8 array) to float64."""
    return _TABLE[np.asarray(bits, dtype=np.uint8)]


def float_to_e4m3(x) -> np.ndarray:
    """Encode floats as e4m3 bit patterns: round to nearest even, saturate to +-448, NaN -> 0x7f."""
    x = np.asarray(x, dtype=np.float64)
    mag = np.abs(x)
    with np.errstate(divide="ignore"):
        k = np.floor(np.log2(np.where(mag > 0, mag, 1.0)))
    step = np.ldexp(1.0, (np.maximum(k, -6) - 3).astype(np.int64))   # spacing at |x|
    q = np.rint(mag / step) * step                                    # rint: ties to even
    q = np.minimum(q, E4M3_MAX)
    code = np.searchsorted(_POSITIVE, q).astype(np.uint8)
    code = np.where(np.signbit(x), code | 0x80, code).astype(np.uint8)
    return np.where(np.isnan(x), np.uint8(0x7F), code).astype(np.uint8)


def gather_sequence(cache, b, length, block_table=None, layout="hnd"):
    """Keys (or values) ``[0, length)`` of sequence ``b`` as a ``(Hkv, length, D)`` array.

    ``cache`` is ``(pages, Hkv, page_size, D)`` for ``layout="hnd"`` or
    ``(pages, page_size, Hkv, D)`` for ``"nhd"``; without a block table page
    ``b`` holds sequence ``b``.
    """
    c = cache if layout == "hnd" else np.swapaxes(cache, 1, 2)
    page_size = c.shape[2]
    if block_table is None:
        return c[b, :, :length, :]
    rows = np.arange(length)
    pages = np.asarray(block_table)[b, rows // page_size]
    return c[pages, :, rows % page_size, :].transpose(1, 0, 2)


def decode_kv_reference(q, k_cache, v_cache, seq_lens=None, *, block_table=None, layout="hnd",
                        scale=None, k_scale=1.0, v_scale=1.0, kv_format=None):
    """Float64 decode of ``q`` (B, Hq, D) over a cache; returns ``(out (B, Hq, D), lse (B, Hq))``.

    ``kv_format="e4m3"`` means the caches hold e4m3 bit patterns (uint8);
    otherwise they hold floating-point values.
    """
    q = np.asarray(q, dtype=np.float64)
    B, Hq, D = q.shape
    c = k_cache if layout == "hnd" else np.swapaxes(k_cache, 1, 2)
    if seq_lens is None:
        seq_lens = np.full(B, c.shape[2], dtype=np.int64)
    out = np.zeros((B, Hq, D), dtype=np.float64)
    lse = np.full((B, Hq), -np.inf, dtype=np.float64)
    for b in range(B):
        n = int(seq_lens[b])
        if n == 0:
            continue
        k = gather_sequence(k_cache, b, n, block_table, layout)
        v = gather_sequence(v_cache, b, n, block_table, layout)
        if kv_format == "e4m3":
            k, v = e4m3_to_float(k), e4m3_to_float(v)
        k = np.asarray(k, dtype=np.float64) * float(k_scale)
        v = np.asarray(v, dtype=np.float64) * float(v_scale)
        qb = q[b][:, None, :]
        gqa = Hq != k.shape[0]
        out[b] = reference_sdpa(qb, k, v, scale=scale, enable_gqa=gqa)[:, 0, :]
        lse[b] = reference_lse(qb, k, scale=scale, enable_gqa=gqa)[:, 0]
    return out, lse
