#!/usr/bin/env python3
"""Build libssa_b200.so (the C-ABI SSA attention library) for sm_100a, in-tree.

    python luciole-1b_b200/build.py [--verbose-ptxas] [--force]

Every ``csrc/*.cu`` is compiled with ``nvcc -gencode arch=compute_100a,code=sm_100a`` into
``_build/*.o`` (incrementally, in parallel) and linked into ``libssa_b200.so`` next to this
file. The CUDA runtime is linked statically; the driver API (``cuTensorMapEncodeTiled``) is
reached through ``cudaGetDriverEntryPoint``, so the library needs no libcuda at link time.
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
REPO = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libssa_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _flags(verbose_ptxas: bool) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                "-I", str(REPO / "include"), "-I", str(CSRC), "--expt-relaxed-constexpr"]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def _deps(src: Path) -> list[Path]:
    return [src] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        [REPO / "include" / "ssa_b200.h"]


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in _deps(src))


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    cc = nvcc()
    jobs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        if force or verbose_ptxas or _stale(o, s):
            jobs.append((s, o))

    def compile_one(so):
        s, o = so
        cmd = [cc] + _flags(verbose_ptxas) + ["-c", str(s), "-o", str(o)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return s, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for s, r in ex.map(compile_one, jobs):
            out = (r.stdout + r.stderr).strip()
            if r.returncode != 0:
                failed.append(s.name)
                print(f"[build] FAILED {s.name}\n{out}", file=sys.stderr)
            elif out and (verbose_ptxas or not quiet):
                print(f"[build] {s.name}\n{out}", file=sys.stderr)
    if failed:
        raise RuntimeError(f"nvcc failed for {failed}")
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [cc] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", str(LIB)] + \
            [str(o) for o in objs] + ["-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
        if not quiet:
            print(f"[build] linked {LIB}", file=sys.stderr)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    build(force=a.force, verbose_ptxas=a.verbose_ptxas)


if __name__ == "__main__":
    main()
