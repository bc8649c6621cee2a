"""NumPy restatement of the reference SDPA forward (oracle; test infrastructure).

Two algorithms are restated here:

* :func:`reference_sdpa` -- the float64 oracle of
  ``src/portable_attention/reference.py:56-163``: upcast to float64
  (``:135-137``), scores ``Q K^T * scale`` (``:139``), top-left causal
  ``tril`` (``:141-144``), boolean keep-mask / additive mask (``:145-149``),
  max-shifted softmax whose fully-masked rows come out exactly zero
  (``:154-160``), ``@ V`` and a cast to the query dtype (``:162``).
* :func:`fused_sdpa` -- the native-precision CPU backend of
  ``src/portable_attention/fused.py:115-218``: the same math in
  ``result_type(q, k, v, float-mask, float32)`` (``:178-184``). This is the
  algorithm the ``cpu_baseline`` leg of ``bench.py`` times.

Validation (``reference.py:110-128``, ``fused.py:155-172``) raises the same
exception types with the same messages, because callers and tests match on
them.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "expand_kv_for_gqa",
    "fused_sdpa",
    "reference_sdpa",
    "softmax_rows",
    "validate_sdpa_args",
]


def expand_kv_for_gqa(query, key, value):
    """Repeat each key/value head ``Hq // Hkv`` times along axis -3.

    Restates ``reference.py:20-53`` (identical copy at ``fused.py:51-83``):
    query head ``h`` attends to key/value head ``h // (Hq // Hkv)``.
    """
    if min(query.ndim, key.ndim, value.ndim) < 3:
        raise ValueError(
            "enable_gqa=True requires a head dimension: query, key, and value "
            "must each have at least 3 dims (*, H, S, E)."
        )
    hq, hk, hv = query.shape[-3], key.shape[-3], value.shape[-3]
    if hk != hv:
        raise ValueError(f"key/value head dims differ: {hk} vs {hv}.")
    if hq == 0 or hk == 0 or hq % hk:
        raise ValueError(
            f"query head count {hq} must be a positive multiple of the "
            f"key/value head count {hk} for grouped-query attention."
        )
    group = hq // hk
    if group == 1:
        return key, value
    return np.repeat(key, group, axis=-3), np.repeat(value, group, axis=-3)


def validate_sdpa_args(query, key, value, attn_mask, dropout_p, is_causal, enable_gqa, backend_label):
    """Argument checks of ``reference.py:110-128`` in the same order.

    Returns the (possibly GQA-expanded) ``key, value``. ``backend_label`` only
    changes the dropout message, as the two reference backends word it
    differently (``reference.py:111-114`` vs ``fused.py:156-158``).
    """
    if dropout_p != 0.0:
        raise NotImplementedError(
            f"dropout_p is not supported by the {backend_label} backend; pass dropout_p=0.0."
        )
    if is_causal and attn_mask is not None:
        raise ValueError("Pass either is_causal=True or attn_mask, not both.")
    if query.ndim < 2 or key.ndim < 2 or value.ndim < 2:
        raise ValueError("query, key, and value must each have at least 2 dims.")
    if enable_gqa:
        key, value = expand_kv_for_gqa(query, key, value)
    if query.shape[-1] != key.shape[-1]:
        raise ValueError(
            f"query/key embedding dims differ: {query.shape[-1]} vs {key.shape[-1]}."
        )
    if key.shape[-2] != value.shape[-2]:
        raise ValueError(
            f"key/value sequence dims differ: {key.shape[-2]} vs {value.shape[-2]}."
        )
    return key, value


def _apply_masks(scores, attn_mask, is_causal, compute_dtype):
    """Causal tril (top-left aligned) or explicit mask, as ``reference.py:141-149``."""
    if is_causal:
        rows, cols = scores.shape[-2:]
        keep = np.tril(np.ones((rows, cols), dtype=bool))
        return np.where(keep, scores, -np.inf)
    if attn_mask is not None:
        if attn_mask.dtype == np.bool_:
            return np.where(attn_mask, scores, -np.inf)
        return scores + attn_mask.astype(compute_dtype)
    return scores


def softmax_rows(scores):
    """Max-shifted softmax over the last axis with exact-zero dead rows.

    Restates ``reference.py:151-160``: a row whose max is not finite is shifted
    by 0, and a row whose exp-sum is 0 (every key masked) is defined as 0.
    """
    peak = np.max(scores, axis=-1, keepdims=True)
    peak = np.where(np.isfinite(peak), peak, 0.0)
    w = np.exp(scores - peak)
    total = np.sum(w, axis=-1, keepdims=True)
    out = np.zeros_like(w)
    np.divide(w, total, out=out, where=total > 0)
    return out


def reference_sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, *,
                   scale=None, enable_gqa=False):
    """Float64 oracle forward (``reference.py:56-163``); output in ``query.dtype``."""
    key, value = validate_sdpa_args(query, key, value, attn_mask, dropout_p, is_causal,
                                    enable_gqa, "CPU reference")
    if scale is None:
        scale = 1.0 / np.sqrt(query.shape[-1])
    q64 = query.astype(np.float64)
    k64 = key.astype(np.float64)
    v64 = value.astype(np.float64)
    scores = np.matmul(q64, np.swapaxes(k64, -1, -2)) * scale
    scores = _apply_masks(scores, attn_mask, is_causal, np.float64)
    probs = softmax_rows(scores)
    return np.matmul(probs, v64).astype(query.dtype)


def fused_sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, *,
               scale=None, enable_gqa=False):
    """Native-precision forward of ``fused.py:115-218`` (BLAS pinning left to the caller).

    The compute dtype is the widest of q/k/v/float-mask with float16 promoted to
    float32 (``fused.py:178-184``); the scale stays a Python float so it does
    not promote float32 scores (``fused.py:187-190``).
    """
    key, value = validate_sdpa_args(query, key, value, attn_mask, dropout_p, is_causal,
                                    enable_gqa, "fused CPU")
    dtypes = [query.dtype, key.dtype, value.dtype]
    if attn_mask is not None and attn_mask.dtype != np.bool_:
        dtypes.append(attn_mask.dtype)
    cdt = np.result_type(*dtypes, np.float32)
    q = query.astype(cdt, copy=False)
    k = key.astype(cdt, copy=False)
    v = value.astype(cdt, copy=False)
    s = float(1.0 / np.sqrt(q.shape[-1])) if scale is None else scale
    scores = np.matmul(q, np.swapaxes(k, -1, -2)) * s
    scores = _apply_masks(scores, attn_mask, is_causal, cdt)
    probs = softmax_rows(scores)
    return np.matmul(probs, v).astype(query.dtype, copy=False)


def reference_lse(query, key, attn_mask=None, is_causal=False, *, scale=None, enable_gqa=False):
    """Float64 natural-log log-sum-exp of the masked, scaled scores per query row.

    Not a reference function: the reference keeps no LSE. It is the quantity
    the CUDA forward saves for the backward and the ring merge, defined on the
    same scores as :func:`reference_sdpa`; fully-masked rows give ``-inf``.
    """
    if enable_gqa:
        key, _ = expand_kv_for_gqa(query, key, key)
    if scale is None:
        scale = 1.0 / np.sqrt(query.shape[-1])
    scores = np.matmul(query.astype(np.float64), np.swapaxes(key.astype(np.float64), -1, -2)) * scale
    scores = _apply_masks(scores, attn_mask, is_causal, np.float64)
    peak = np.max(scores, axis=-1, keepdims=True)
    peak = np.where(np.isfinite(peak), peak, 0.0)
    with np.errstate(divide="ignore"):
        return (np.log(np.sum(np.exp(scores - peak), axis=-1, keepdims=True)) + peak)[..., 0]
