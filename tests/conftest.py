"""Shared pytest setup: import paths, the ``gpu`` marker and golden fixtures.

``-m "not gpu"`` runs everywhere (oracle against the golden vectors, host
logic, library symbol table). ``-m gpu`` needs a CUDA device and the built
``libpa_b200.so``; those tests compare the CUDA path with the golden vectors
and the oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (ROOT, ROOT / "portable-attention_b200", GOLDEN):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and libpa_b200.so")


@pytest.fixture(scope="session")
def golden_conformance():
    return dict(np.load(GOLDEN / "conformance.npz", allow_pickle=False))


@pytest.fixture(scope="session")
def golden_extra():
    return dict(np.load(GOLDEN / "extra.npz", allow_pickle=False))


@pytest.fixture(scope="session")
def golden_rows():
    return dict(np.load(GOLDEN / "workload_rows.npz", allow_pickle=False))


@pytest.fixture(scope="session")
def reference_package():
    """The real reference package: ``$PA_REFERENCE_SRC``, else ``oracle/_ref``
    (byte-compiled by ``oracle/build_ref.py``, which ``__graft_entry__.build()`` runs)."""
    from oracle import build_ref

    pa = build_ref.import_reference()
    if pa is None:
        pytest.skip("reference package not built (python oracle/build_ref.py)")
    return pa


@pytest.fixture(scope="session")
def cuda_backend():
    """The CUDA SdpaBackend; fails (not skips) when the GPU path cannot run."""
    import pa_b200

    assert pa_b200.available(), "gpu test without a usable CUDA device / libpa_b200.so"
    return pa_b200.scaled_dot_product_attention
