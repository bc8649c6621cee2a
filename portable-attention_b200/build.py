"""Build libpa_b200.so in-tree with nvcc for sm_100a.

Usage: ``python portable-attention_b200/build.py [--jobs N] [--force]``.

Every ``csrc/*.cu`` is compiled to an object under ``_build/`` (skipped when
the object is newer than its source and the shared headers), then linked
into ``pa_b200/libpa_b200.so`` against the static CUDA runtime. The library
resolves ``cuTensorMapEncodeTiled`` through the runtime's driver entry point
and loads NCCL with dlopen on first use of the ring (only its header is
needed here), so it links neither libcuda nor libnccl and builds on a host
without a GPU.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
BUILD = ROOT / "_build"
OUT = HERE / "pa_b200" / "libpa_b200.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libpa_b200")
    return cand


def nccl_flags() -> tuple[list[str], list[str]]:
    """Include flags for nccl.h (NCCL itself is loaded at run time) and link flags."""
    inc = [p for p in ("/usr/include", "/usr/local/cuda/include") if Path(p, "nccl.h").exists()]
    if not inc:
        raise RuntimeError("nccl.h not found")
    return [f"-I{inc[0]}"], ["-ldl"]


def compile_one(src: Path, force: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    deps = [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")]
    if not force and obj.exists() and obj.stat().st_mtime >= max(p.stat().st_mtime for p in deps):
        return obj, ""
    inc, _ = nccl_flags()
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", *inc, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        results = list(ex.map(lambda s: compile_one(s, force), sources))
    objs = [r[0] for r in results]
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    _, libs = nccl_flags()
    newest = max(o.stat().st_mtime for o in objs)
    if force or not OUT.exists() or OUT.stat().st_mtime < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(OUT), *map(str, objs), *libs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
    return OUT


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
