"""Build the reference's own CUDA extension, unmodified, as a cross-oracle.

TEST INFRASTRUCTURE ONLY.  Nothing in ``mamba_b200`` imports this file or its output.

The reference (nmquan1503/Mamba) ships no CPU implementation and no golden vectors,
so its CUDA extension ``selective_scan`` (csrc/selective_scan/selective_scan.cpp,
forward_kernel.cu, backward_kernel.cu) is the only thing that can pin the CPU oracle.
This recipe compiles those three source files where they lie, with the nvcc flags of
the reference's setup.py:10-30 plus an explicit sm_100a target (the reference has
none and takes the arch from TORCH_CUDA_ARCH_LIST), and writes the module only into
``oracle/_ref/`` (git-ignored, but it travels to the GPU box).  It does not run the
reference's own setup.py / pip build.

Usage:  python oracle/build_ref.py [--ref PATH]   (default: $MAMBA_REFERENCE_ROOT, else a directory
        named `reference` beside this repository)
"""
from __future__ import annotations

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def reference_root() -> str:
    """$MAMBA_REFERENCE_ROOT, else a directory named `reference` beside this repository."""
    repo = os.path.dirname(HERE)
    return os.environ.get("MAMBA_REFERENCE_ROOT", os.path.join(os.path.dirname(repo), "reference"))


def build(ref_root: str | None = None, verbose: bool = False) -> str | None:
    ref_root = ref_root or reference_root()
    src = os.path.join(ref_root, "csrc", "selective_scan")
    if not os.path.isdir(src):
        print(f"[build_ref] reference sources not found at {src}; skipping", file=sys.stderr)
        return None
    os.makedirs(OUT, exist_ok=True)
    from torch.utils import cpp_extension

    srcs = [os.path.join(src, f) for f in ("selective_scan.cpp", "forward_kernel.cu", "backward_kernel.cu")]
    mod = cpp_extension.load(
        name="selective_scan",
        sources=srcs,
        extra_include_paths=[src],
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=[
            "-O3", "-std=c++17", "--use_fast_math", "--expt-relaxed-constexpr",
            "--expt-extended-lambda",
            "-gencode", "arch=compute_100a,code=sm_100a",
        ],
        build_directory=OUT,
        verbose=verbose,
        is_python_module=True,
    )
    path = getattr(mod, "__file__", None)
    print(f"[build_ref] built {path}")
    return path


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="reference tree (default: $MAMBA_REFERENCE_ROOT, else "
                                                  "../reference beside this repository)")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    # cpp_extension otherwise appends every arch in TORCH_CUDA_ARCH_LIST
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    build(a.ref, a.v)
