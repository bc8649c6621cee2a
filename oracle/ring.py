"""NumPy simulation of n-rank ring attention (oracle; test infrastructure).

The reference has no distributed code, so nothing in it pins this file; it is
pinned by equality with :func:`oracle.sdpa.reference_sdpa` and
:func:`oracle.vjp.reference_vjp` on the gathered sequence
(``tests/test_ring_host.py``). It replays, in float64, exactly the
step-by-step data movement of the GPU ring: rank ``r`` holds the key/value
shard of rank ``(r - t) mod n`` in step ``t``, computes the pairs a schedule
function gives it, merges partial outputs by log-sum-exp, and (backward)
passes fp64 dK/dV accumulators along with the key/value shard, one extra hop
bringing them home.
"""

from __future__ import annotations

import numpy as np

__all__ = ["block_attention", "block_grads", "simulate_ring"]


def block_attention(q, k, causal, scale):
    """Unnormalised block: (row max-shifted weights, lse) of q against k (float64)."""
    s = np.einsum("...id,...jd->...ij", q, k) * scale
    if causal:
        s = np.where(np.tril(np.ones(s.shape[-2:], dtype=bool)), s, -np.inf)
    m = np.max(s, axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    w = np.exp(s - m)
    tot = np.sum(w, axis=-1, keepdims=True)
    with np.errstate(divide="ignore"):
        lse = np.log(tot) + m
    return w, tot, lse[..., 0]


def block_grads(q, k, v, do, o, lse, causal, scale):
    """dQ, dK, dV contributions of one (query chunk, key chunk) pair (float64)."""
    s = np.einsum("...id,...jd->...ij", q, k) * scale
    if causal:
        s = np.where(np.tril(np.ones(s.shape[-2:], dtype=bool)), s, -np.inf)
    p = np.where(np.isfinite(lse[..., None]), np.exp(s - lse[..., None]), 0.0)
    dp = np.einsum("...id,...jd->...ij", do, v)
    delta = np.sum(do * o, axis=-1, keepdims=True)
    ds = p * (dp - delta)
    dq = scale * np.einsum("...ij,...jd->...id", ds, k)
    dk = scale * np.einsum("...ij,...id->...jd", ds, q)
    dv = np.einsum("...ij,...id->...jd", p, do)
    return dq, dk, dv


def simulate_ring(q, k, v, n, pairs, do=None, scale=None):
    """Run the ring over ``n`` simulated ranks; shards are (..., 2C, D) per rank.

    ``q, k, v, do`` are lists of per-rank shards (same head counts; float64
    math). ``pairs(n, r, t)`` yields (query slot, key slot, causal). Returns
    per-rank (out, lse) and, when ``do`` is given, per-rank (dq, dk, dv).
    """
    if scale is None:
        scale = 1.0 / np.sqrt(q[0].shape[-1])
    c = q[0].shape[-2] // 2
    slot = lambda x, s: x[..., s * c:(s + 1) * c, :]  # noqa: E731
    outs, lses = [], []
    for r in range(n):
        acc_o = [np.zeros(slot(q[r], s).shape[:-1] + (v[r].shape[-1],)) for s in (0, 1)]
        acc_l = [np.full(slot(q[r], s).shape[:-1], -np.inf) for s in (0, 1)]
        for t in range(n):
            src = (r - t) % n
            for qs, ks, causal in pairs(n, r, t):
                w, tot, lse = block_attention(slot(q[r], qs).astype(np.float64),
                                              slot(k[src], ks).astype(np.float64), causal, scale)
                part = np.divide(w @ slot(v[src], ks).astype(np.float64), tot,
                                 out=np.zeros(acc_o[qs].shape), where=tot > 0)
                m = np.maximum(acc_l[qs], lse)
                m_safe = np.where(np.isfinite(m), m, 0.0)
                wa = np.where(np.isfinite(acc_l[qs]), np.exp(acc_l[qs] - m_safe), 0.0)
                wb = np.where(np.isfinite(lse), np.exp(lse - m_safe), 0.0)
                den = wa + wb
                acc_o[qs] = np.divide(acc_o[qs] * wa[..., None] + part * wb[..., None], den[..., None],
                                      out=acc_o[qs].copy(), where=den[..., None] > 0)
                with np.errstate(divide="ignore"):
                    acc_l[qs] = np.where(den > 0, m_safe + np.log(den), -np.inf)
        outs.append(np.concatenate(acc_o, axis=-2))
        lses.append(np.concatenate(acc_l, axis=-1))
    if do is None:
        return outs, lses
    # Backward: dK/dV accumulators start at their owner and move with the K/V.
    held = {r: [np.zeros(k[r].shape), np.zeros(v[r].shape)] for r in range(n)}  # keyed by source
    dqs = [np.zeros(q[r].shape) for r in range(n)]
    for t in range(n):
        for r in range(n):
            src = (r - t) % n
            for qs, ks, causal in pairs(n, r, t):
                gq, gk, gv = block_grads(slot(q[r], qs).astype(np.float64), slot(k[src], ks).astype(np.float64),
                                         slot(v[src], ks).astype(np.float64), slot(do[r], qs).astype(np.float64),
                                         slot(outs[r], qs), slot(lses[r][..., None], qs)[..., 0], causal, scale)
                dqs[r][..., qs * c:(qs + 1) * c, :] += gq
                held[src][0][..., ks * c:(ks + 1) * c, :] += gk
                held[src][1][..., ks * c:(ks + 1) * c, :] += gv
    return outs, lses, [(dqs[r], held[r][0], held[r][1]) for r in range(n)]
