"""Builds the reference's own hash-grid encoder (TEST INFRASTRUCTURE ONLY).

NilKel/nest-splatting ships `gridencoder/` (a torch CUDA extension:
gridencoder/src/gridencoder.cu, bindings.cpp, gridencoder.h). Its forward
kernel (`kernel_grid`, gridencoder.cu:88-242) evaluates, per level, exactly the
per-level lookup that the rasterizer's `query_feature` performs
(submodules/diff-surfel-rasterization/cuda_rasterizer/hashgrid.h:7-40 and
:128-212: same fast_hash primes, dense/hashed index rule, level scale and
trilinear weights); its backward kernels (`kernel_grid_backward`, :246-338, and
`kernel_input_backward`, :341-367) give the table gradient and dL/dx of the same
lookup. Unlike the rasterizer it needs no glm, so it builds here.

This script compiles those sources unmodified, where they lie in the reference
checkout, with the reference's own nvcc flags (gridencoder/setup.py:7-15) plus
the sm_100a target, into oracle/_ref/gridencoder/ (git-ignored; it travels with
the repository snapshot to the GPU box, where the reference checkout does not
exist). tests/golden/make_gridencoder_golden.py runs it there to write golden
vectors; nothing in the product loads it.

Usage: python oracle/build_ref.py [reference_root]   (default: $NEST_REFERENCE or
the reference checkout next to the build container's repository).
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "gridencoder"
NAME = "_gridencoder_ref"
DEFAULT_REF = os.environ.get("NEST_REFERENCE", "/root/reference")

# gridencoder/setup.py:7-15, with the B200 target added.
NVCC_FLAGS = ["-O3", "-std=c++17", "--expt-relaxed-constexpr",
              "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
              "-U__CUDA_NO_HALF2_OPERATORS__",
              "-gencode=arch=compute_100a,code=sm_100a"]
C_FLAGS = ["-O3", "-std=c++17"]


def so_path() -> Path | None:
    hits = sorted(OUT.glob(NAME + "*.so"))
    return hits[0] if hits else None


def build(ref_root: str = DEFAULT_REF, verbose: bool = False) -> Path | None:
    """Compiles the reference gridencoder into oracle/_ref/gridencoder/ (once:
    an existing module is kept; the build takes several minutes, most of it in
    torch's headers).

    Returns the built module path, or None when the reference checkout is
    absent (as on the GPU box, which only uses the prebuilt module)."""
    src = Path(ref_root) / "gridencoder" / "src"
    if so_path() is not None or not (src / "gridencoder.cu").exists():
        return so_path()
    from torch.utils.cpp_extension import load

    OUT.mkdir(parents=True, exist_ok=True)
    load(name=NAME, sources=[str(src / "gridencoder.cu"), str(src / "bindings.cpp")],
         extra_cflags=C_FLAGS, extra_cuda_cflags=NVCC_FLAGS, build_directory=str(OUT),
         verbose=verbose, with_cuda=True)
    # keep only the module: the objects and ninja files would travel to the GPU box too
    for p in OUT.iterdir():
        if p.suffix != ".so":
            p.unlink()
    return so_path()


def load_module():
    """Imports the prebuilt reference module (needs `import torch` first)."""
    import torch  # noqa: F401  (the module links against torch's libraries)

    path = so_path()
    if path is None:
        raise FileNotFoundError(f"{OUT}: reference gridencoder not built (python oracle/build_ref.py)")
    loader = importlib.machinery.ExtensionFileLoader(NAME, str(path))
    spec = importlib.util.spec_from_loader(NAME, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    p = build(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF, verbose=True)
    print(p)
