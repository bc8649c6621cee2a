"""Build the reference package into ``oracle/_ref`` (test infrastructure).

The reference (portable-attention) is a pure-Python package, so its "build"
is a byte-compile: every module of ``src/portable_attention`` is compiled,
from the sources where they lie, into one code bundle in ``oracle/_ref/``.
Nothing is modified. The output is
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
checkout at ``/root/reference``. :func:`import_reference` loads the result.
"""

from __future__ import annotations

import importlib
import importlib.abc
import importlib.util
import marshal
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
PACKAGE = "portable_attention"


BUNDLE = OUT / (PACKAGE + ".codebundle")


def build(reference_root: str | os.PathLike | None = None) -> Path | None:
    """Byte-compile the reference package into ``oracle/_ref``; ``None`` if absent.

    The code objects of every module go into one file (``marshal`` format, a
    map from module name to compiled code), which :func:`import_reference`
    loads through its own importer.
    """
    root = Path(reference_root or os.environ.get("PA_REFERENCE_ROOT", "/root/reference"))
    src = root / "src" / PACKAGE
    if not (src / "__init__.py").exists():
        return None
    if OUT.exists():
        shutil.rmtree(OUT)
    OUT.mkdir(parents=True)
    codes = {}
    for py in sorted(src.glob("*.py")):
        name = PACKAGE if py.stem == "__init__" else f"{PACKAGE}.{py.stem}"
        code = compile(py.read_bytes(), f"{PACKAGE}/{py.name}", "exec", dont_inherit=True)
        codes[name] = marshal.dumps(code)
    BUNDLE.write_bytes(marshal.dumps({"python": sys.version_info[:2], "modules": codes}))
    (OUT / "SOURCE.txt").write_text(f"byte-compiled from {src} by oracle/build_ref.py\n"
                                    f"python {sys.version.split()[0]}\n")
    return BUNDLE


class _BundleFinder(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    """Imports the reference package from the code bundle written by :func:`build`."""

    def __init__(self, modules):
        self.modules = modules

    def find_spec(self, fullname, path=None, target=None):
        if fullname not in self.modules:
            return None
        return importlib.util.spec_from_loader(fullname, self, is_package=fullname == PACKAGE)

    def create_module(self, spec):
        return None

    def exec_module(self, module):
        if module.__name__ == PACKAGE:
            module.__path__ = []
        module.__file__ = f"<{BUNDLE.name}:{module.__name__}>"
        exec(marshal.loads(self.modules[module.__name__]), module.__dict__)


def import_reference():
    """Import and return the reference package (``None`` when it is not available).

    ``$PA_REFERENCE_SRC`` (a ``src`` folder of a reference checkout) wins;
    otherwise the bundle :func:`build` wrote, when it matches this Python.
    """
    if PACKAGE in sys.modules:
        return sys.modules[PACKAGE]
    env = os.environ.get("PA_REFERENCE_SRC")
    if env and (Path(env) / PACKAGE / "__init__.py").exists():
        if env not in sys.path:
            sys.path.insert(0, env)
        return importlib.import_module(PACKAGE)
    if not BUNDLE.exists():
        return None
    blob = marshal.loads(BUNDLE.read_bytes())
    if tuple(blob.get("python", ())) != sys.version_info[:2]:
        return None
    # One finder, for this bundle (a finder left by an earlier bundle is replaced).
    sys.meta_path[:] = [f for f in sys.meta_path if not isinstance(f, _BundleFinder)]
    sys.meta_path.insert(0, _BundleFinder(blob["modules"]))
    return importlib.import_module(PACKAGE)


if __name__ == "__main__":
    got = build(sys.argv[1] if len(sys.argv) > 1 else None)
    print(got if got else "reference checkout not found; nothing built")
