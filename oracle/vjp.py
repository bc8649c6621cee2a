"""Float64 VJP of the reference SDPA forward (oracle; test infrastructure).

The reference has no backward pass, so nothing in it can pin this file; it is
pinned instead by central finite differences of
:func:`oracle.sdpa.reference_sdpa` in ``tests/test_oracle.py``.

With ``S = scale * Q K^T (+ mask)``, ``P = softmax(S)`` (dead rows 0) and
``O = P V``, the cotangent ``dO`` gives::

    dV = P^T dO
    dP = dO V^T
    dS = P * (dP - rowsum(dO * O))
    dQ = scale * dS K
    dK = scale * dS^T Q

Under grouped-query attention the expanded key/value heads share storage, so
``dK`` / ``dV`` are summed over each group of ``Hq // Hkv`` query heads.
"""

from __future__ import annotations

import numpy as np

from .sdpa import _apply_masks, expand_kv_for_gqa, softmax_rows

__all__ = ["reference_vjp"]


def reference_vjp(query, key, value, dout, attn_mask=None, is_causal=False, *, scale=None,
                  enable_gqa=False):
    """Return ``(dq, dk, dv)`` in float64 for the forward of ``reference.py:56-163``."""
    hkv = key.shape[-3] if enable_gqa else None
    if enable_gqa:
        key, value = expand_kv_for_gqa(query, key, value)
    if scale is None:
        scale = 1.0 / np.sqrt(query.shape[-1])
    q = query.astype(np.float64)
    k = key.astype(np.float64)
    v = value.astype(np.float64)
    do = dout.astype(np.float64)
    scores = np.matmul(q, np.swapaxes(k, -1, -2)) * scale
    scores = _apply_masks(scores, attn_mask, is_causal, np.float64)
    p = softmax_rows(scores)
    o = np.matmul(p, v)
    dv = np.matmul(np.swapaxes(p, -1, -2), do)
    dp = np.matmul(do, np.swapaxes(v, -1, -2))
    delta = np.sum(do * o, axis=-1, keepdims=True)
    ds = p * (dp - delta)
    dq = scale * np.matmul(ds, k)
    dk = scale * np.matmul(np.swapaxes(ds, -1, -2), q)
    if enable_gqa and hkv is not None and hkv != query.shape[-3]:
        group = query.shape[-3] // hkv
        lead = dk.shape[:-3]
        dk = dk.reshape(*lead, hkv, group, *dk.shape[-2:]).sum(axis=-3)
        dv = dv.reshape(*lead, hkv, group, *dv.shape[-2:]).sum(axis=-3)
    return dq, dk, dv
