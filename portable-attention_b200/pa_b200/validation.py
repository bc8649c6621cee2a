"""Argument checks of the portable-attention SDPA contract.

Same checks, same order, same exception types and messages as the reference
backends (``src/portable_attention/reference.py:110-128`` and the grouped-query
rules of ``reference.py:36-49``), because callers and the reference's tests
match on those messages. Only the dropout message names this backend.
"""

from __future__ import annotations

__all__ = ["check_gqa_heads", "validate"]


def check_gqa_heads(query, key, value) -> int:
    """Return the grouped-query group size ``Hq // Hkv`` or raise like ``reference.py:36-49``."""
    if query.ndim < 3 or key.ndim < 3 or value.ndim < 3:
        raise ValueError(
            "enable_gqa=True requires a head dimension: query, key, and value "
            "must each have at least 3 dims (*, H, S, E)."
        )
    hq, hk = query.shape[-3], key.shape[-3]
    if hk != value.shape[-3]:
        raise ValueError(f"key/value head dims differ: {hk} vs {value.shape[-3]}.")
    if hq == 0 or hk == 0 or hq % hk != 0:
        raise ValueError(
            f"query head count {hq} must be a positive multiple of the "
            f"key/value head count {hk} for grouped-query attention."
        )
    return hq // hk


def validate(query, key, value, attn_mask, dropout_p, is_causal, enable_gqa) -> int:
    """Validate one call; return the grouped-query group size (1 without GQA)."""
    if dropout_p != 0.0:
        raise NotImplementedError(
            "dropout_p is not supported by the CUDA backend; pass dropout_p=0.0."
        )
    if is_causal and attn_mask is not None:
        raise ValueError("Pass either is_causal=True or attn_mask, not both.")
    if query.ndim < 2 or key.ndim < 2 or value.ndim < 2:
        raise ValueError("query, key, and value must each have at least 2 dims.")
    group = check_gqa_heads(query, key, value) if enable_gqa else 1
    if query.shape[-1] != key.shape[-1]:
        raise ValueError(
            f"query/key embedding dims differ: {query.shape[-1]} vs {key.shape[-1]}."
        )
    if key.shape[-2] != value.shape[-2]:
        raise ValueError(
            f"key/value sequence dims differ: {key.shape[-2]} vs {value.shape[-2]}."
        )
    return group
