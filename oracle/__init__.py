"""CPU oracle for the scaled-dot-product-attention hot path (test infrastructure).

This package is the *checker*, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it. The CUDA backend in ``pa_b200`` never routes
through it and fails loudly when its native library is missing.

Contents (each function cites the reference file:line it restates; paths are
relative to the portable-attention project root):

* :mod:`oracle.sdpa` -- the float64 ``reference`` algorithm
  (``src/portable_attention/reference.py:20-163``) and the native-precision
  ``fused`` algorithm (``src/portable_attention/fused.py:115-218``), with the
  reference's validation messages.
* :mod:`oracle.vjp` -- a float64 VJP (dQ, dK, dV) of the same forward. The
  reference has no backward, so this is pinned by central finite differences
  in ``tests/test_oracle.py`` instead of by reference vectors.
* :mod:`oracle.conformance` -- the canonical conformance matrix and the
  per-case acceptance rule (``src/portable_attention/conformance.py:66-298``).
* :mod:`oracle.ring` -- an n-rank NumPy simulation of ring attention with a
  log-sum-exp merge, used to check the host-side ring schedule.
* :mod:`oracle.build_ref` -- byte-compiles the real reference package into
  ``oracle/_ref`` (git-ignored, carried with the working tree) and imports it
  from there, so the reference's own conformance kit and CPU backends run
  where no reference checkout exists (tests, and bench.py's CPU baseline).

Pinning: ``tests/golden/make_golden.py`` imports the real reference package and
writes its outputs to ``tests/golden/*.npz``; ``tests/test_oracle.py`` checks
this restatement against those vectors.
"""
