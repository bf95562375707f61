"""Build libactune_b200.so (sm_100a) in-tree with nvcc.

    python -m actune_b200.build [--force] [--verbose-ptxas]

Each csrc/*.cu is compiled to an object with relocatable device code (the
device error word is shared by all kernels), then nvcc device-links them into
one shared library next to this file.  The CUDA runtime is linked statically so
the library only needs the driver at run time.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libactune_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC,-O2",
              "--expt-relaxed-constexpr", "-Xcudafe", "--diag_suppress=177"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (needed to build libactune_b200.so)")


def sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None,
          out: Path | None = None) -> Path:
    headers = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    srcs = sources()
    lib = Path(out) if out else LIB
    build_dir = BUILD if out is None else lib.parent / ("_build_" + lib.stem)
    build_dir.mkdir(exist_ok=True, parents=True)
    objs = [build_dir / (s.stem + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(o, [s, *headers, Path(__file__)])]
    cc = nvcc()

    def compile_one(so):
        s, o = so
        cmd = [cc, *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(s), "-o", str(o)]
        if verbose_ptxas:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {s.name}:\n{r.stdout}\n{r.stderr}")
        return s.name, r.stderr

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            for name, err in ex.map(compile_one, todo):
                if verbose_ptxas and err:
                    print(f"== {name}\n{err}")
    if force or todo or _stale(lib, objs):
        cmd = [cc, *ARCH, "-shared", "-rdc=true", "-cudart", "static", "-o", str(lib), *map(str, objs),
               "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
    return lib


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--out", default=None, help="output library path (default: in-tree libactune_b200.so)")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas, jobs=a.jobs, out=a.out))


if __name__ == "__main__":
    main()
