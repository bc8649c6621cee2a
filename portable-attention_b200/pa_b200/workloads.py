"""Seeded synthetic inputs for the five attention workloads this backend is measured on.

Each generator draws ``numpy.random.default_rng(seed).standard_normal`` in the
order query, key, value (then any extra draws), in float64, and casts to the
workload's dtype -- the same recipe the portable-attention conformance kit uses
for its cases (``src/portable_attention/conformance.py:110-127``). The
float64 stream of ``standard_normal`` is chunk-invariant, so large tensors are
produced in slabs through one reusable float64 buffer instead of one multi-GB
temporary.

Workloads (shapes are ``(batch, heads, seq, head_dim)``):

``fp32_unmasked``  fp32 q,k,v (4, 8, 512, 64), seed 0, non-causal, no mask.
``fp16_causal_gqa`` fp16 q (8, 32, 4096, 128), k,v (8, 8, 4096, 128), seed 1,
                   causal, grouped-query (4 query heads per key/value head).
``fp16_masked_cross`` fp16 q (16, 16, 1024, 64), k,v (16, 16, 2048, 64), seed 2;
                   boolean key-padding mask (16, 1, 1024, 2048) keeping the first
                   ``n_b`` keys of batch row ``b``, ``n_b`` drawn after v as
                   ``rng.integers(1024, 2049, size=16)``.
``fp16_decode_gqa`` fp16 q (64, 32, 1, 128), k,v (64, 8, 32768, 128), all
                   ``N(0,1) * 0.5``, seed 3, grouped-query.
``fp16_long_causal`` fp16 q,k,v (1, 32, 131072, 128), seed 4, causal; upstream
                   gradient dO (same shape) from seed 5.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

__all__ = ["WORKLOADS", "Workload", "draw", "make"]

_SLAB = 1 << 24  # float64 values per generation slab (128 MiB)


def draw(gen, shape, dtype, scale=1.0, out=None):
    """Fill a ``shape`` array of ``dtype`` from ``gen.standard_normal`` slab by slab."""
    n = int(np.prod(shape))
    res = np.empty(n, dtype=dtype) if out is None else out.reshape(-1)
    buf = np.empty(min(n, _SLAB), dtype=np.float64)
    pos = 0
    while pos < n:
        m = min(_SLAB, n - pos)
        gen.standard_normal(out=buf[:m])
        if scale != 1.0:
            buf[:m] *= scale
        res[pos:pos + m] = buf[:m]
        pos += m
    return res.reshape(shape)


@dataclass(frozen=True)
class Workload:
    name: str
    q_shape: tuple
    kv_shape: tuple
    dtype: str
    seed: int
    is_causal: bool = False
    enable_gqa: bool = False
    masked: bool = False
    scale_inputs: float = 1.0
    backward: bool = False

    @property
    def flops_fwd(self) -> float:
        """Algorithmic forward FLOPs: 4 * B * Hq * Lq * Lk * D, halved when causal."""
        b, hq, lq, d = self.q_shape
        lk = self.kv_shape[2]
        f = 4.0 * b * hq * lq * lk * d
        return f / 2 if self.is_causal else f

    @property
    def flops_bwd(self) -> float:
        """Algorithmic backward FLOPs: 2.5x the forward."""
        return 2.5 * self.flops_fwd

    @property
    def io_bytes(self) -> int:
        """Bytes of q, k, v read and out written once (no mask)."""
        es = np.dtype(self.dtype).itemsize
        q = int(np.prod(self.q_shape))
        kv = int(np.prod(self.kv_shape))
        return es * (2 * q + 2 * kv)


WORKLOADS = {
    w.name: w
    for w in (
        Workload("fp32_unmasked", (4, 8, 512, 64), (4, 8, 512, 64), "float32", 0),
        Workload("fp16_causal_gqa", (8, 32, 4096, 128), (8, 8, 4096, 128), "float16", 1,
                 is_causal=True, enable_gqa=True),
        Workload("fp16_masked_cross", (16, 16, 1024, 64), (16, 16, 2048, 64), "float16", 2,
                 masked=True),
        Workload("fp16_decode_gqa", (64, 32, 1, 128), (64, 8, 32768, 128), "float16", 3,
                 enable_gqa=True, scale_inputs=0.5),
        Workload("fp16_long_causal", (1, 32, 131072, 128), (1, 32, 131072, 128), "float16", 4,
                 is_causal=True, backward=True),
    )
}


def make(name, *, batch_rows=None):
    """Return the seeded inputs of workload ``name`` as a dict of NumPy arrays.

    Keys: ``q``, ``k``, ``v`` and, where the workload has them, ``mask`` (bool)
    and ``dout``. ``batch_rows`` (a ``slice``) keeps only those batch rows of
    every tensor after drawing the full stream, so a sampled check sees exactly
    the values the full workload does.
    """
    w = WORKLOADS[name]
    dt = np.dtype(w.dtype)
    gen = np.random.default_rng(w.seed)
    q = draw(gen, w.q_shape, dt, w.scale_inputs)
    k = draw(gen, w.kv_shape, dt, w.scale_inputs)
    v = draw(gen, w.kv_shape, dt, w.scale_inputs)
    res = {"q": q, "k": k, "v": v}
    if w.masked:
        keep = gen.integers(1024, 2049, size=w.q_shape[0])
        lq, lk = w.q_shape[2], w.kv_shape[2]
        cols = np.arange(lk)
        mask = np.broadcast_to((cols[None, :] < keep[:, None])[:, None, None, :],
                               (w.q_shape[0], 1, lq, lk))
        res["mask"] = np.ascontiguousarray(mask)
        res["keep"] = keep
    if w.backward:
        res["dout"] = draw(np.random.default_rng(w.seed + 1), w.q_shape, dt, 1.0)
    if batch_rows is not None:
        res = {key: (val[batch_rows] if key != "keep" else val[batch_rows])
               for key, val in res.items()}
    return res
