"""Build the in-tree native extensions.

``python -m mmltk_b200.build`` compiles

* ``mmltk_b200/_kernels*.so`` from ``csrc/kernels`` for sm_100a only
  (``-gencode arch=compute_100a,code=sm_100a``; torch's own arch list is
  bypassed because the flag is given explicitly), and
* ``mmltk_b200/_native*.so`` from ``csrc/host`` (plain C++17, no CUDA).

Both land next to the Python sources (``build_ext --inplace``) so a snapshot
of the repository carries them to a GPU machine.  nvcc cross-compiles, so no
GPU is needed to build.
"""
from __future__ import annotations

import glob
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-Xptxas", "-warn-spills",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-DNDEBUG"]


def extensions():
    from torch.utils.cpp_extension import CppExtension, CUDAExtension

    kern_src = sorted(p for p in glob.glob(os.path.join("csrc", "kernels", "*.cu")) +
                      glob.glob(os.path.join("csrc", "kernels", "*.cpp")) if "noalloc" not in p)
    host_src = sorted(glob.glob(os.path.join("csrc", "host", "*.cpp")))
    inc = [os.path.join(ROOT, "csrc", "include"), os.path.join(ROOT, "csrc", "kernels")]
    return [
        CppExtension("mmltk_b200._native", host_src, include_dirs=inc + [os.path.join(ROOT, "csrc", "host")],
                     extra_compile_args={"cxx": CXX_FLAGS}, extra_link_args=["-lpthread", "-lz"]),
        CUDAExtension("mmltk_b200._kernels", kern_src, include_dirs=inc,
                      extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS}),
    ]


NOALLOC_LIB = os.path.join(ROOT, "mmltk_b200", "libmmltk_noalloc.so")


def build_noalloc(verbose: bool = False) -> str:
    """Plain C-ABI library with the allocation-free MSDeformAttn backward
    (``mmltk_msda_bwd_noalloc``, see csrc/kernels/msda_noalloc.h).  It is kept
    out of the torch extension so its fixed scratch array is only reserved by
    processes that load it."""
    import subprocess

    srcs = [os.path.join(ROOT, "csrc", "kernels", f) for f in ("msda.cu", "msda_noalloc.cu")]
    newest = max(os.path.getmtime(p) for p in srcs + [os.path.join(ROOT, "csrc", "kernels", "launch_api.h"),
                                                       os.path.join(ROOT, "csrc", "kernels", "common.cuh"),
                                                       os.path.join(ROOT, "csrc", "kernels", "msda_noalloc.h")])
    if os.path.exists(NOALLOC_LIB) and os.path.getmtime(NOALLOC_LIB) >= newest:
        return NOALLOC_LIB
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC", "-cudart", "shared", "-I", os.path.join(ROOT, "csrc", "kernels"), *srcs,
           "-o", NOALLOC_LIB]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return NOALLOC_LIB


def build(verbose: bool = False, jobs: int | None = None) -> None:
    from setuptools import setup
    from torch.utils.cpp_extension import BuildExtension

    os.environ.setdefault("MAX_JOBS", str(jobs or os.cpu_count() or 8))
    cwd = os.getcwd()
    os.chdir(ROOT)
    try:
        args = ["build_ext", "--inplace"]
        if not verbose:
            args.insert(0, "-q")
        setup(name="mmltk_b200_native", ext_modules=extensions(),
              cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
              script_args=args)
    finally:
        os.chdir(cwd)
    build_noalloc(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
