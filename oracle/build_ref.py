"""Build the reference package into ``oracle/_ref`` (test infrastructure).

The reference (portable-attention) is a pure-Python package, so its "build"
is a byte-compile: every module of ``src/portable_attention`` is compiled,
from the sources where they lie, to a sourceless ``.pyc`` in
``oracle/_ref/portable_attention/``. Nothing is modified. The output is
git-ignored (it is the reference's code, not this repository's) but travels
with the working tree, so the reference's own ``reference`` / ``fused``
backends, its conformance kit and its thread helpers can be imported on a
machine that has no reference checkout:

* ``tests/`` run ``portable_attention.assert_conforms`` on the CUDA backend;
* ``bench.py`` times the reference's CPU backends for ``cpu_baseline`` and
  ``--impl reference``.

An offline ``pip install`` of the reference is not possible here: its build
backend (hatchling) is not available without a package index.

Usage::

    python oracle/build_ref.py [REFERENCE_ROOT]

``REFERENCE_ROOT`` defaults to ``$PA_REFERENCE_ROOT`` or the read-only
checkout at ``/root/reference``. :func:`reference_path` finds the result.
"""

from __future__ import annotations

import os
import py_compile
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
PACKAGE = "portable_attention"


def build(reference_root: str | os.PathLike | None = None) -> Path | None:
    """Byte-compile the reference package into ``oracle/_ref``; ``None`` if absent."""
    root = Path(reference_root or os.environ.get("PA_REFERENCE_ROOT", "/root/reference"))
    src = root / "src" / PACKAGE
    if not (src / "__init__.py").exists():
        return None
    dst = OUT / PACKAGE
    if dst.exists():
        shutil.rmtree(dst)
    dst.mkdir(parents=True)
    for py in sorted(src.glob("*.py")):
        py_compile.compile(str(py), cfile=str(dst / (py.stem + ".pyc")), doraise=True,
                           invalidation_mode=py_compile.PycInvalidationMode.UNCHECKED_HASH)
    stamp = dst.parent / "SOURCE.txt"
    stamp.write_text(f"byte-compiled from {src} by oracle/build_ref.py\n"
                     f"python {sys.version.split()[0]}\n")
    return dst


def reference_path() -> Path | None:
    """Folder to put on ``sys.path`` to import the reference package, or ``None``.

    ``$PA_REFERENCE_SRC`` (a ``src`` folder of a reference checkout) wins;
    otherwise ``oracle/_ref`` when :func:`build` has filled it.
    """
    env = os.environ.get("PA_REFERENCE_SRC")
    if env and (Path(env) / PACKAGE / "__init__.py").exists():
        return Path(env)
    if (OUT / PACKAGE / "__init__.pyc").exists():
        return OUT
    return None


def import_reference():
    """Import and return the reference package (``None`` when it is not available)."""
    path = reference_path()
    if path is None:
        return None
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))
    import importlib

    return importlib.import_module(PACKAGE)


if __name__ == "__main__":
    got = build(sys.argv[1] if len(sys.argv) > 1 else None)
    print(got if got else "reference checkout not found; nothing built")
