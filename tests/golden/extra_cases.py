"""Extra edge cases beyond the conformance matrix (pure NumPy, seeded).

Shared by ``make_golden.py`` (which stores the reference outputs for them in
``extra.npz``) and the tests (which regenerate the same inputs from the seed,
so the fixture holds only outputs and a fingerprint of the inputs).
"""

from __future__ import annotations

import numpy as np


def extra_cases():
    g = np.random.default_rng(1234)

    def n(*s, dt=np.float32):
        return g.standard_normal(s).astype(dt)

    yield "causal-L<S", (n(2, 5, 8), n(2, 9, 8), n(2, 9, 4)), {"is_causal": True}
    yield "causal-L>S", (n(2, 9, 8), n(2, 5, 8), n(2, 5, 4)), {"is_causal": True}
    m = g.random((3, 1, 5, 7)) > 0.5
    yield "bool-mask-head-broadcast", (n(3, 4, 5, 8), n(3, 4, 7, 8), n(3, 4, 7, 6)), {"attn_mask": m}
    bias = g.standard_normal((5, 7)).astype(np.float32)
    bias[2] = -np.inf
    yield "additive-dead-row", (n(2, 5, 8), n(2, 7, 8), n(2, 7, 8)), {"attn_mask": bias}
    yield "f64-additive-on-f32", (n(2, 5, 8), n(2, 7, 8), n(2, 7, 4)), {
        "attn_mask": g.standard_normal((2, 5, 7))}
    yield "mixed-q32-kv64", (n(2, 4, 6, 8), n(2, 4, 6, 8, dt=np.float64),
                             n(2, 4, 6, 4, dt=np.float64)), {}
    yield "2d-unbatched-f64", (n(33, 20, dt=np.float64), n(41, 20, dt=np.float64),
                               n(41, 3, dt=np.float64)), {"scale": 0.7}
    yield "5d-lead-f32", (n(2, 2, 3, 6, 10), n(2, 2, 3, 11, 10), n(2, 2, 3, 11, 5)), {}
    h = np.float16
    yield "tc-f16-d64-gqa-causal", (n(2, 4, 200, 64, dt=h), n(2, 2, 200, 64, dt=h),
                                    n(2, 2, 200, 64, dt=h)), {"is_causal": True, "enable_gqa": True}
    yield "tc-f16-d128-ragged", (n(1, 3, 130, 128, dt=h), n(1, 3, 257, 128, dt=h),
                                 n(1, 3, 257, 128, dt=h)), {}
    yield "tc-f16-d128-causal-L<S", (n(1, 2, 100, 128, dt=h), n(1, 2, 300, 128, dt=h),
                                     n(1, 2, 300, 128, dt=h)), {"is_causal": True}
    km = g.random((2, 1, 150, 333)) > 0.3
    km[0, 0, 7] = False
    yield "tc-f16-d64-bool-mask", (n(2, 3, 150, 64, dt=h), n(2, 3, 333, 64, dt=h),
                                   n(2, 3, 333, 64, dt=h)), {"attn_mask": km}
    ab = (g.standard_normal((1, 2, 140, 260)) * 2).astype(h)
    ab[0, 1, 3, :] = -np.inf
    yield "tc-f16-d128-additive", (n(1, 2, 140, 128, dt=h), n(1, 2, 260, 128, dt=h),
                                   n(1, 2, 260, 128, dt=h)), {"attn_mask": ab}
    yield "decode-f16-gqa", (n(3, 8, 1, 128, dt=h) * h(0.5), n(3, 2, 3000, 128, dt=h) * h(0.5),
                             n(3, 2, 3000, 128, dt=h) * h(0.5)), {"enable_gqa": True}
    yield "decode-f16-d64", (n(2, 4, 1, 64, dt=h), n(2, 4, 777, 64, dt=h),
                             n(2, 4, 777, 64, dt=h)), {}
