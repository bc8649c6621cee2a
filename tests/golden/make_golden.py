"""Regenerate the golden vectors in this directory from the real reference package.

Run from the repository root in a checkout that has the portable-attention
sources (read-only is fine)::

    PA_REFERENCE_SRC=/root/reference/src python tests/golden/make_golden.py

It imports ``portable_attention`` from ``PA_REFERENCE_SRC`` and records, with
the reference's own ``reference`` and ``fused`` backends:

* ``conformance.npz`` -- inputs and both backends' outputs for the 26 cases of
  ``portable_attention.conformance.conformance_cases()``;
* ``extra.npz`` -- reference outputs (and an input fingerprint) for the extra
  edge cases of ``extra_cases.py`` (L != S
  causal alignment, broadcast masks, -inf additive rows, mixed dtypes, shapes
  the tensor-core and decode kernels take);
* ``workload_rows.npz`` -- reference outputs on sampled rows of the full-size
  workloads of ``pa_b200.workloads`` (a slice of query rows against every key,
  with an explicit lower-triangular mask slice for causal rows);
* ``messages.json`` -- the exact exception type and text for invalid calls.

Nothing on the GPU side reads the reference: only these files travel.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, os.environ.get("PA_REFERENCE_SRC", "/root/reference/src"))
sys.path.insert(0, str(ROOT / "portable-attention_b200"))

import portable_attention as pa  # noqa: E402
from portable_attention.conformance import conformance_cases  # noqa: E402

from pa_b200 import workloads  # noqa: E402

sys.path.insert(0, str(HERE))
from extra_cases import extra_cases  # noqa: E402

REF = pa.get_backend("reference")
FUSED = pa.get_backend("fused")


def conformance():
    blob = {}
    names = []
    for i, case in enumerate(conformance_cases()):
        q, k, v = case.make_inputs()
        kw = dict(case.kwargs)
        names.append(case.name)
        blob[f"{i}_q"], blob[f"{i}_k"], blob[f"{i}_v"] = q, k, v
        blob[f"{i}_ref"] = REF(q, k, v, **kw)
        blob[f"{i}_fused"] = FUSED(q, k, v, **kw)
        if "attn_mask" in kw:
            blob[f"{i}_mask"] = kw["attn_mask"]
    blob["names"] = np.array(names)
    np.savez_compressed(HERE / "conformance.npz", **blob)


def extra():
    blob = {}
    names = []
    for i, (name, (q, k, v), kw) in enumerate(extra_cases()):
        names.append(name)
        blob[f"{i}_ref"] = REF(q, k, v, **kw)
        blob[f"{i}_fingerprint"] = np.array([float(x.astype(np.float64).sum()) for x in (q, k, v)])
    blob["names"] = np.array(names)
    np.savez_compressed(HERE / "extra.npz", **blob)


def _rows(name, picks):
    """Reference output rows for (batch, head, row0, nrows) picks of workload ``name``."""
    w = workloads.WORKLOADS[name]
    x = workloads.make(name)
    group = w.q_shape[1] // w.kv_shape[1]
    out = {}
    for b, hq, r0, nr in picks:
        q = x["q"][b, hq, r0:r0 + nr]
        k = x["k"][b, hq // group]
        v = x["v"][b, hq // group]
        kw = {}
        if w.is_causal:
            rows = np.arange(r0, r0 + nr)[:, None]
            kw["attn_mask"] = np.arange(k.shape[0])[None, :] <= rows
        elif w.masked:
            kw["attn_mask"] = x["mask"][b, 0, r0:r0 + nr]
        out[f"{name}|{b}|{hq}|{r0}|{nr}"] = REF(q, k, v, **kw)
    fp = {f"{name}|fingerprint": np.array([x["q"].ravel()[:4].astype(np.float64),
                                           x["k"].ravel()[-4:].astype(np.float64),
                                           x["v"].ravel()[-4:].astype(np.float64)])}
    return {**out, **fp}


def workload_rows():
    blob = {}
    blob.update(_rows("fp32_unmasked", [(0, 0, 0, 16), (3, 7, 496, 16), (2, 5, 250, 8)]))
    blob.update(_rows("fp16_causal_gqa", [(0, 0, 0, 8), (0, 5, 1000, 8), (7, 31, 4088, 8),
                                          (3, 17, 2047, 4)]))
    blob.update(_rows("fp16_masked_cross", [(0, 0, 0, 8), (5, 3, 500, 8), (15, 15, 1016, 8)]))
    blob.update(_rows("fp16_decode_gqa", [(0, h, 0, 1) for h in (0, 1, 5, 31)] + [(63, 7, 0, 1)]))
    np.savez_compressed(HERE / "workload_rows.npz", **blob)


def long_rows():
    blob = _rows("fp16_long_causal", [(0, 0, 0, 4), (0, 9, 70000, 4), (0, 31, 131068, 4)])
    np.savez_compressed(HERE / "long_rows.npz", **blob)


def messages():
    g = np.random.default_rng(0)
    z = np.zeros
    calls = {
        "ndim": ((z(4), z((3, 4)), z((3, 4))), {}),
        "embed": ((z((5, 8)), z((6, 7)), z((6, 3))), {}),
        "seq": ((z((5, 8)), z((6, 8)), z((7, 3))), {}),
        "dropout": ((z((2, 4, 8)), z((2, 4, 8)), z((2, 4, 8))), {"dropout_p": 0.1}),
        "causal+mask": ((z((4, 4, 8)), z((4, 4, 8)), z((4, 4, 8))),
                        {"attn_mask": np.ones((4, 4), bool), "is_causal": True}),
        "gqa-ndim": ((z((5, 8)), z((7, 8)), z((7, 4))), {"enable_gqa": True}),
        "gqa-multiple": ((z((2, 8, 5, 8)), z((2, 3, 7, 8)), z((2, 3, 7, 4))), {"enable_gqa": True}),
        "gqa-kv-heads": ((z((2, 8, 5, 8)), z((2, 2, 7, 8)), z((2, 4, 7, 4))), {"enable_gqa": True}),
        "gqa-zero": ((z((2, 0, 5, 8)), z((2, 2, 7, 8)), z((2, 2, 7, 4))), {"enable_gqa": True}),
    }
    del g
    res = {}
    for key, (args, kw) in calls.items():
        for label, fn in (("reference", REF), ("fused", FUSED)):
            try:
                fn(*args, **kw)
                res[f"{key}|{label}"] = None
            except Exception as exc:  # noqa: BLE001
                res[f"{key}|{label}"] = [type(exc).__name__, str(exc)]
    (HERE / "messages.json").write_text(json.dumps(res, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    what = sys.argv[1:] or ["conformance", "extra", "messages", "workload_rows", "long_rows"]
    for step in what:
        globals()[step]()
        print("wrote", step)
