"""The conformance matrix and acceptance rule (oracle; test infrastructure).

Restates ``src/portable_attention/conformance.py``: the per-dtype tolerances
(``:66-70``), the seeded input factory (``:110-127``), the 26-case matrix
(``:130-247``: 12 unmasked shape x dtype cases, scaled and causal per dtype,
boolean / additive / fully-masked masks, four GQA head splits and GQA+causal)
and the acceptance rule of ``check_case`` (``:254-298``: shape, dtype,
finiteness, ``allclose`` in float64 against the oracle, exact zeros on
fully-masked rows). Case names and seeds are kept identical because test ids
and the inputs they draw are the interface being matched.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .sdpa import reference_sdpa

__all__ = ["TOLERANCES", "Case", "cases", "check"]

TOLERANCES = {
    np.dtype(np.float64): (1e-11, 1e-11),
    np.dtype(np.float32): (1e-4, 1e-5),
    np.dtype(np.float16): (2e-3, 2e-3),
}


@dataclass(frozen=True)
class Case:
    name: str
    shapes: tuple
    dtype: type
    seed: int
    kwargs: dict = field(default_factory=dict)

    def inputs(self):
        gen = np.random.default_rng(self.seed)
        dt = np.dtype(self.dtype)
        return tuple(gen.standard_normal(s).astype(dt) for s in self.shapes)


def _qkv(lead, length, source, e, ev):
    return ((*lead, length, e), (*lead, source, e), (*lead, source, ev))


def cases():
    """The 26 canonical cases, in the reference's order."""
    out = []
    dtypes = (np.float64, np.float32, np.float16)
    shape_rows = (((), 4, 4, 8, 8), ((3,), 5, 7, 8, 4), ((2, 3), 5, 7, 6, 4),
                  ((1, 8), 16, 16, 64, 64))
    for dt in dtypes:
        for lead, length, source, e, ev in shape_rows:
            out.append(Case(f"unmasked-{np.dtype(dt).name}-{lead}-{length}x{source}",
                            _qkv(lead, length, source, e, ev), dt, 1))
    for dt in dtypes:
        name = np.dtype(dt).name
        out.append(Case(f"scaled-{name}", ((2, 3, 5, 8), (2, 3, 7, 8), (2, 3, 7, 4)), dt, 2,
                        {"scale": 0.3}))
        out.append(Case(f"causal-{name}", ((2, 4, 6, 8), (2, 4, 6, 8), (2, 4, 6, 4)), dt, 3,
                        {"is_causal": True}))
    keep = np.random.default_rng(40).random((5, 7)) > 0.3
    out.append(Case("bool-mask", ((2, 5, 8), (2, 7, 8), (2, 7, 4)), np.float32, 4,
                    {"attn_mask": keep}))
    bias = np.random.default_rng(50).standard_normal((5, 7)).astype(np.float32)
    out.append(Case("additive-mask", ((2, 5, 8), (2, 7, 8), (2, 7, 4)), np.float32, 5,
                    {"attn_mask": bias}))
    dead = np.ones((3, 5, 7), dtype=bool)
    dead[0] = False
    out.append(Case("fully-masked-rows", ((3, 5, 8), (3, 7, 8), (3, 7, 4)), np.float32, 6,
                    {"attn_mask": dead}))
    for hq, hkv in ((8, 2), (6, 3), (4, 1), (4, 4)):
        out.append(Case(f"gqa-{hq}q-{hkv}kv", ((2, hq, 5, 8), (2, hkv, 7, 8), (2, hkv, 7, 4)),
                        np.float64, 7, {"enable_gqa": True}))
    out.append(Case("gqa-causal", ((2, 8, 6, 8), (2, 2, 6, 8), (2, 2, 6, 4)), np.float64, 8,
                    {"enable_gqa": True, "is_causal": True}))
    return out


def check(backend, case, want=None):
    """Return ``(passed, detail)`` for one case, with ``conformance.py:254-298``'s rule."""
    q, k, v = case.inputs()
    if want is None:
        want = reference_sdpa(q, k, v, **case.kwargs)
    try:
        got = backend(q, k, v, **case.kwargs)
    except Exception as exc:  # noqa: BLE001 -- a raise on a valid case is a failure
        return False, f"backend raised {type(exc).__name__}: {exc}"
    if got.shape != want.shape:
        return False, f"shape {got.shape} != oracle {want.shape}"
    if got.dtype != q.dtype:
        return False, f"dtype {got.dtype} != query dtype {q.dtype} (silent cast)"
    if not np.all(np.isfinite(got)):
        return False, "output contains non-finite values"
    rtol, atol = TOLERANCES[q.dtype]
    g64, w64 = got.astype(np.float64), want.astype(np.float64)
    if not np.allclose(g64, w64, rtol=rtol, atol=atol):
        return False, f"value mismatch vs oracle (max abs diff {np.max(np.abs(g64 - w64)):.3e})"
    dead_rows = np.all(want == 0.0, axis=-1)
    if np.any(dead_rows) and not np.array_equal(got[dead_rows], want[dead_rows]):
        return False, "fully-masked rows are not exactly zero"
    return True, ""
