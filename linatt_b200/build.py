"""Build the sm_100a shared library ``linatt_b200/libkata_b200.so`` from ``linatt_b200/csrc``.

Each ``.cu`` file is compiled to an object in parallel with
``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3``, then the objects are linked
into one shared library that exports the C ABI declared in ``include/kata_b200.h``.  The build
is incremental: an object is rebuilt only when its source or any header is newer than it.
The library is written in-tree so that it travels with the repository snapshot.

Usage: ``python -m linatt_b200.build [-j N] [--force] [--ptxas-verbose]``
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "libkata_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build linatt_b200")
    return cand


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(obj: Path, src: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return t < src.stat().st_mtime or t < newest_header


def _compile(src: Path, obj: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    cmd = [nvcc(), *ARCH, *CFLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
    return src, r.stderr


def build(jobs: int | None = None, force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> Path:
    """Compile every CUDA source for sm_100a and link ``libkata_b200.so``; returns its path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    todo = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, src, newest_header):
            todo.append((src, obj))
    jobs = jobs or max(1, min(len(todo), os.cpu_count() or 1))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = [ex.submit(_compile, s, o, verbose_ptxas) for s, o in todo]
            for f in cf.as_completed(futs):
                src, log = f.result()
                if not quiet:
                    print(f"[build] compiled {src.name}", file=sys.stderr)
                if verbose_ptxas and log:
                    print(log, file=sys.stderr)
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    lib = build(a.jobs, a.force, a.ptxas_verbose, quiet=False)
    print(lib)


if __name__ == "__main__":
    main()
