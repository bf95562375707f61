"""Build the reference's own CUDA kernels as a GPU-side checker.  TEST INFRASTRUCTURE ONLY.

    python -m oracle.build_ref          # in the build container, where the reference is mounted

Compiles, from the reference's sources where they lie, the three native
extensions its Python loaders JIT-build (paths relative to the reference root):

* ``actune/kernels/grouped_native.cu``  -- the group-64 W{2,4}xA{2,4} linear
  (loader: actune/kernels/grouped.py:97-105, flags -O3);
* ``actune/kernels/grouped_big_m.cu``   -- its 13 tuned tile geometries
  (loader: actune/kernels/tuning.py, flags -O3);
* ``actune/kernels/native_s4_extension.cpp`` + ``native_s4_extension_kernel.cu``
  -- the per-row A4 W{2,4}A4 linears (loader: actune/kernels/wxa4_native.py:
  103-118, flags -O3 --use_fast_math).

The reference builds them for the GPU it runs on; here they are cross-compiled
for sm_100a with the same flags, through torch.utils.cpp_extension as the
reference does, and the modules are written to ``oracle/_ref/`` (git-ignored; the
built .so files travel to the GPU box, the reference sources do not).  Nothing
of the reference is copied: only the compiled modules are kept.

``load(name)`` imports a built module (tests only).  When a module is absent the
caller skips the comparison and says so.
"""
from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
REFERENCE = Path(os.environ.get("ACTUNE_REFERENCE_ROOT", "/root/reference"))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

# module name -> (sources relative to the reference root, extra CUDA flags)
MODULES = {
    "ref_grouped_native": (["actune/kernels/grouped_native.cu"], ["-O3"]),
    "ref_grouped_big_m": (["actune/kernels/grouped_big_m.cu"], ["-O3"]),
    "ref_native_s4": (["actune/kernels/native_s4_extension.cpp", "actune/kernels/native_s4_extension_kernel.cu"],
                      ["-O3", "--use_fast_math"]),
}


def build(names=None, verbose=False) -> dict:
    """Build the named modules (all by default); returns {name: path or error text}."""
    from torch.utils.cpp_extension import load

    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    OUT.mkdir(exist_ok=True)
    results = {}
    for name in names or MODULES:
        srcs, flags = MODULES[name]
        paths = [REFERENCE / s for s in srcs]
        if not all(p.exists() for p in paths):
            results[name] = "reference sources not present"
            continue
        bdir = OUT / f"_build_{name}"
        bdir.mkdir(exist_ok=True)
        try:
            load(name=name, sources=[str(p) for p in paths], extra_cuda_cflags=[*flags, *ARCH],
                 extra_cflags=["-O3"], build_directory=str(bdir), verbose=verbose)
            so = next(bdir.glob(f"{name}*.so"))
            target = OUT / so.name
            target.write_bytes(so.read_bytes())
            results[name] = str(target)
        except Exception as exc:  # a build failure is reported, not raised
            results[name] = f"build failed: {str(exc).splitlines()[-1] if str(exc) else type(exc).__name__}"
    return results


def load_path(name):
    """Path of the built module `name` in oracle/_ref, or None."""
    hits = sorted(OUT.glob(f"{name}*.so"))
    return hits[0] if hits else None


def load(name):
    """Import a module built by build() from oracle/_ref, or None when absent."""
    path = load_path(name)
    if path is None:
        return None
    import torch  # noqa: F401  (the modules link against torch)
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    for k, v in build(sys.argv[1:] or None, verbose="-v" in sys.argv).items():
        print(f"{k}: {v}")
