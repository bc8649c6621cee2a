"""The CPU oracle, pinned against vectors produced by the real reference package.

``tests/golden/make_golden.py`` ran portable-attention's own ``reference`` and
``fused`` backends; these tests require the NumPy restatement in ``oracle/`` to
reproduce those outputs, validation messages and workload rows. The float64
VJP has no reference counterpart and is pinned by central finite differences.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from extra_cases import extra_cases
from oracle import conformance as oc
from oracle.sdpa import fused_sdpa, reference_lse, reference_sdpa
from oracle.vjp import reference_vjp
from conftest import GOLDEN

CASES = oc.cases()


def test_case_matrix_matches_reference_names(golden_conformance):
    assert [c.name for c in CASES] == list(golden_conformance["names"])
    assert len(CASES) == 26


@pytest.mark.parametrize("idx", range(26), ids=[c.name for c in CASES])
def test_oracle_reproduces_reference_and_fused(idx, golden_conformance):
    g = golden_conformance
    case = CASES[idx]
    q, k, v = case.inputs()
    for name, arr in (("q", q), ("k", k), ("v", v)):
        np.testing.assert_array_equal(arr, g[f"{idx}_{name}"])
    if f"{idx}_mask" in g:
        np.testing.assert_array_equal(case.kwargs["attn_mask"], g[f"{idx}_mask"])
    ref = reference_sdpa(q, k, v, **case.kwargs)
    assert ref.dtype == g[f"{idx}_ref"].dtype
    np.testing.assert_array_equal(ref, g[f"{idx}_ref"])
    fused = fused_sdpa(q, k, v, **case.kwargs)
    np.testing.assert_allclose(fused.astype(np.float64), g[f"{idx}_fused"].astype(np.float64),
                               rtol=1e-6, atol=1e-7)


def test_extra_cases_match_reference(golden_extra):
    g = golden_extra
    names = list(g["names"])
    for i, (name, (q, k, v), kw) in enumerate(extra_cases()):
        assert names[i] == name
        fp = np.array([float(x.astype(np.float64).sum()) for x in (q, k, v)])
        np.testing.assert_array_equal(fp, g[f"{i}_fingerprint"], err_msg=name)
        got = reference_sdpa(q, k, v, **kw)
        np.testing.assert_array_equal(got, g[f"{i}_ref"], err_msg=name)


def test_validation_messages_match_reference():
    golden = json.loads((GOLDEN / "messages.json").read_text())
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
    for key, (args, kw) in calls.items():
        for label, fn in (("reference", reference_sdpa), ("fused", fused_sdpa)):
            want = golden[f"{key}|{label}"]
            with pytest.raises(Exception) as info:
                fn(*args, **kw)
            assert [type(info.value).__name__, str(info.value)] == want, (key, label)


def test_workload_rows_cheap_configs(golden_rows):
    """Full-size seeded inputs reproduce the fingerprints and oracle rows of the fixture."""
    from pa_b200 import workloads

    for name in ("fp32_unmasked", "fp16_masked_cross"):
        x = workloads.make(name)
        fp = np.array([x["q"].ravel()[:4].astype(np.float64), x["k"].ravel()[-4:].astype(np.float64),
                       x["v"].ravel()[-4:].astype(np.float64)])
        np.testing.assert_array_equal(fp, golden_rows[f"{name}|fingerprint"])
        for key in golden_rows:
            parts = key.split("|")
            if parts[0] != name or parts[1] == "fingerprint":
                continue
            b, h, r0, nr = map(int, parts[1:])
            kw = {}
            if name == "fp16_masked_cross":
                kw["attn_mask"] = x["mask"][b, 0, r0:r0 + nr]
            got = reference_sdpa(x["q"][b, h, r0:r0 + nr], x["k"][b, h], x["v"][b, h], **kw)
            np.testing.assert_array_equal(got, golden_rows[key])


def test_masked_cross_mask_is_key_padding():
    from pa_b200 import workloads

    x = workloads.make("fp16_masked_cross")
    keep = x["keep"]
    assert keep.min() >= 1024 and keep.max() <= 2048
    for b in (0, 7, 15):
        row = x["mask"][b, 0, 0]
        assert row[:keep[b]].all() and not row[keep[b]:].any()
        assert (x["mask"][b, 0] == row).all()


def _fd_grad(f, x, eps=1e-6):
    g = np.zeros_like(x)
    it = np.nditer(x, flags=["multi_index"])
    for _ in it:
        i = it.multi_index
        old = x[i]
        x[i] = old + eps
        fp = f()
        x[i] = old - eps
        fm = f()
        x[i] = old
        g[i] = (fp - fm) / (2 * eps)
    return g


@pytest.mark.parametrize("kw", [{}, {"is_causal": True}, {"enable_gqa": True},
                                {"attn_mask": "bool"}, {"attn_mask": "add"}, {"scale": 0.37}],
                         ids=["plain", "causal", "gqa", "bool", "additive", "scale"])
def test_vjp_matches_finite_differences(kw):
    rng = np.random.default_rng(3)
    hq, hkv = (4, 2) if kw.get("enable_gqa") else (2, 2)
    q = rng.standard_normal((2, hq, 5, 6))
    k = rng.standard_normal((2, hkv, 7, 6))
    v = rng.standard_normal((2, hkv, 7, 3))
    do = rng.standard_normal((2, hq, 5, 3))
    kw = dict(kw)
    if kw.get("attn_mask") == "bool":
        m = rng.random((5, 7)) > 0.3
        m[1] = False  # one fully-masked row: zero output, zero gradient
        kw["attn_mask"] = m
    elif kw.get("attn_mask") == "add":
        kw["attn_mask"] = rng.standard_normal((2, 1, 5, 7))

    def loss():
        return float(np.sum(reference_sdpa(q, k, v, **kw) * do))

    dq, dk, dv = reference_vjp(q, k, v, do, **kw)
    for got, x in ((dq, q), (dk, k), (dv, v)):
        np.testing.assert_allclose(got, _fd_grad(loss, x), rtol=1e-6, atol=1e-8)


def test_lse_matches_direct_log_sum_exp():
    rng = np.random.default_rng(9)
    q = rng.standard_normal((3, 4, 8))
    k = rng.standard_normal((3, 6, 8))
    m = rng.random((4, 6)) > 0.4
    m[2] = False
    lse = reference_lse(q, k, attn_mask=m)
    s = np.einsum("bie,bje->bij", q, k) / np.sqrt(8)
    with np.errstate(divide="ignore"):
        want = np.log(np.sum(np.where(m, np.exp(s), 0.0), axis=-1))
    np.testing.assert_allclose(lse, want, rtol=1e-12)
    assert np.all(np.isneginf(lse[:, 2]))


# -- the acceptance rule itself catches planted mistakes (planted on the CPU) --

def _ref_backend(q, k, v, **kw):
    return reference_sdpa(q, k, v, **kw)


@pytest.mark.parametrize("mistake,needle", [
    (lambda o: o[..., :1], "shape"),
    (lambda o: o.astype(np.float16), "dtype"),
    (lambda o: np.where(np.arange(o.size).reshape(o.shape) == 0, np.nan, o).astype(o.dtype), "non-finite"),
    (lambda o: o + 1.0, "value mismatch"),
])
def test_acceptance_rule_flags_planted_mistakes(mistake, needle):
    case = oc.Case("probe", ((2, 4, 8), (2, 4, 8), (2, 4, 8)), np.float64, 0)
    ok, detail = oc.check(lambda *a, **kw: mistake(_ref_backend(*a, **kw)), case)
    assert not ok and needle in detail


def test_acceptance_rule_flags_nonzero_dead_rows():
    dead = np.ones((3, 5, 7), dtype=bool)
    dead[0] = False
    case = oc.Case("dead", ((3, 5, 8), (3, 7, 8), (3, 7, 4)), np.float64, 0, {"attn_mask": dead})

    def tiny(q, k, v, **kw):
        out = np.array(_ref_backend(q, k, v, **kw))
        out[0] += 1e-13
        return out

    ok, detail = oc.check(tiny, case)
    assert not ok and "exactly zero" in detail


def test_acceptance_rule_flags_raising_backend():
    case = oc.Case("probe", ((2, 4, 8), (2, 4, 8), (2, 4, 8)), np.float64, 0)

    def boom(*a, **kw):
        raise RuntimeError("boom")

    ok, detail = oc.check(boom, case)
    assert not ok and "backend raised RuntimeError: boom" in detail


def test_reference_bundle_builds_and_imports(tmp_path, monkeypatch):
    """oracle/build_ref.py byte-compiles a package tree into one code bundle and imports it
    through its own finder; a bundle for another Python version is ignored."""
    import marshal
    import sys

    from oracle import build_ref

    src = tmp_path / "ref" / "src" / build_ref.PACKAGE
    src.mkdir(parents=True)
    (src / "__init__.py").write_text("from .mod import answer\n__all__ = ['answer']\n")
    (src / "mod.py").write_text("def answer():\n    return 42\n")
    out = tmp_path / "_ref"
    monkeypatch.setattr(build_ref, "OUT", out)
    monkeypatch.setattr(build_ref, "BUNDLE", out / (build_ref.PACKAGE + ".codebundle"))
    monkeypatch.delenv("PA_REFERENCE_SRC", raising=False)
    saved = {k: sys.modules.pop(k) for k in list(sys.modules) if k.split(".")[0] == build_ref.PACKAGE}
    saved_path = list(sys.meta_path)
    try:
        assert build_ref.build(tmp_path / "ref") == build_ref.BUNDLE
        assert not list(out.rglob("*.py"))            # code objects only, no sources
        pkg = build_ref.import_reference()
        assert pkg.answer() == 42
        # A bundle written by another Python version is not loaded.
        for k in [k for k in sys.modules if k.split(".")[0] == build_ref.PACKAGE]:
            del sys.modules[k]
        sys.meta_path[:] = saved_path
        blob = marshal.loads(build_ref.BUNDLE.read_bytes())
        blob["python"] = (2, 7)
        build_ref.BUNDLE.write_bytes(marshal.dumps(blob))
        assert build_ref.import_reference() is None
        assert build_ref.build(tmp_path / "missing") is None
    finally:
        for k in [k for k in sys.modules if k.split(".")[0] == build_ref.PACKAGE]:
            del sys.modules[k]
        sys.modules.update(saved)
        sys.meta_path[:] = saved_path
