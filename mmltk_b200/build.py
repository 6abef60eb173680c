"""Build the in-tree native extensions.

``python -m mmltk_b200.build`` compiles

* ``mmltk_b200/_kernels*.so`` from ``csrc/kernels`` for sm_100a only
  (``-gencode arch=compute_100a,code=sm_100a``; torch's own arch list is
  bypassed because the flag is given explicitly), and
* ``mmltk_b200/_native*.so`` from ``csrc/host`` (plain C++17, no CUDA);
* ``mmltk_b200/_sdpa_packed*.so`` from ``csrc/cudnn`` (host C++ on the cuDNN graph API);
* with ``--debug-bounds``, also ``mmltk_b200/_kernels_dbg*.so``: the same kernels compiled with
  ``-DMMLTK_DEBUG_BOUNDS=1``, whose index checks record an error code in a device status word
  (``kernels().debug_status()``) instead of trapping; ``MMLTK_DEBUG_BOUNDS=1`` at run time loads
  it in place of ``_kernels``;
* with ``--host-sanitize address,undefined``, the host self-test (``csrc/host/selftest_main.cpp``
  over the torch-free host sources) as an ASan / UBSan executable, ``build/host_selftest_san``.

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


DEBUG_FLAGS = ["-DMMLTK_DEBUG_BOUNDS=1"]


def extensions(debug_bounds: bool = False):
    from torch.utils.cpp_extension import CppExtension, CUDAExtension

    kern_src = sorted(p for p in glob.glob(os.path.join("csrc", "kernels", "*.cu")) +
                      glob.glob(os.path.join("csrc", "kernels", "*.cpp")) if "noalloc" not in p)
    host_src = sorted(p for p in glob.glob(os.path.join("csrc", "host", "*.cpp")) if "selftest" not in p)
    inc = [os.path.join(ROOT, "csrc", "include"), os.path.join(ROOT, "csrc", "kernels")]
    exts = [
        CppExtension("mmltk_b200._native", host_src, include_dirs=inc + [os.path.join(ROOT, "csrc", "host")],
                     extra_compile_args={"cxx": CXX_FLAGS}, extra_link_args=["-lpthread", "-lz"]),
        CUDAExtension("mmltk_b200._kernels", kern_src, include_dirs=inc,
                      extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS}),
    ]
    exts.append(_cudnn_extension(inc))
    if debug_bounds:
        exts.append(CUDAExtension("mmltk_b200._kernels_dbg", kern_src, include_dirs=inc,
                                  extra_compile_args={"cxx": CXX_FLAGS + DEBUG_FLAGS,
                                                      "nvcc": NVCC_FLAGS + DEBUG_FLAGS}))
    return exts


def _cudnn_paths():
    """(frontend include dir, cuDNN include dir, cuDNN library dir) of the cuDNN that torch loads."""
    import site
    for sp in site.getsitepackages():
        fe = os.path.join(sp, "include")
        cd = os.path.join(sp, "nvidia", "cudnn")
        if os.path.exists(os.path.join(fe, "cudnn_frontend.h")) and os.path.isdir(cd):
            return fe, os.path.join(cd, "include"), os.path.join(cd, "lib")
    raise RuntimeError("cudnn_frontend.h / the nvidia-cudnn package not found in site-packages")


def _cudnn_extension(inc):
    """``mmltk_b200._sdpa_packed``: cuDNN SDPA backward into strided (packed) gradient views
    (``csrc/cudnn/sdpa_packed.cpp``), linked against the libcudnn.so.9 that torch loads."""
    from torch.utils.cpp_extension import CUDAExtension
    fe_inc, cudnn_inc, cudnn_lib = _cudnn_paths()
    # The image's g++ resolves -lstdc++ to the static archive (its shared-library link is dangling)
    # and links shared objects with -Bsymbolic, so a library would run its stream / locale code on a
    # private, never-initialised copy of libstdc++ (the cuDNN frontend formats numbers through
    # std::ostream, and that crashed).  The process's shared libstdc++ is named explicitly; hidden
    # visibility keeps the header-only frontend's symbols (libtorch carries its own copy) private.
    return CUDAExtension("mmltk_b200._sdpa_packed", [os.path.join("csrc", "cudnn", "sdpa_packed.cpp")],
                         include_dirs=inc + [fe_inc, cudnn_inc],
                         extra_compile_args={"cxx": CXX_FLAGS + ["-fvisibility=hidden", "-fvisibility-inlines-hidden"],
                                             "nvcc": NVCC_FLAGS},
                         extra_link_args=[f"-L{cudnn_lib}", "-l:libcudnn.so.9", f"-Wl,-rpath,{cudnn_lib}",
                                          "-Wl,--no-as-needed", _shared_libstdcxx(), "-Wl,--as-needed"])


def _shared_libstdcxx() -> str:
    """Path of the shared libstdc++ the Python process itself uses."""
    for d in ("/usr/lib/x86_64-linux-gnu", "/usr/lib64", "/lib/x86_64-linux-gnu"):
        p = os.path.join(d, "libstdc++.so.6")
        if os.path.exists(p):
            return p
    raise RuntimeError("shared libstdc++.so.6 not found")


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


HOST_SELFTEST_SOURCES = ("lsap.cpp", "worker_pool.cpp", "image_io.cpp", "selftest_main.cpp")


def build_host_selftest(sanitize: str = "address,undefined", verbose: bool = False) -> str:
    """ASan / UBSan build of the host self-test (the counterpart of the reference's Dev-build
    sanitizer options, `cmake/mmltk_project_configuration.cmake:72-79`): torch-free host sources plus
    ``csrc/host/selftest_main.cpp``, linked into ``build/host_selftest_san``.  Returns its path."""
    import subprocess

    out_dir = os.path.join(ROOT, "build")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "host_selftest_san")
    srcs = [os.path.join(ROOT, "csrc", "host", f) for f in HOST_SELFTEST_SOURCES]
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", f"-fsanitize={sanitize}",
           "-fno-sanitize-recover=undefined", "-I", os.path.join(ROOT, "csrc", "host"), *srcs, "-o", exe,
           "-lpthread", "-lz"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    return exe


def build(verbose: bool = False, jobs: int | None = None, debug_bounds: bool = False) -> None:
    from setuptools import setup
    from torch.utils.cpp_extension import BuildExtension

    os.environ.setdefault("MAX_JOBS", str(jobs or os.cpu_count() or 8))
    cwd = os.getcwd()
    os.chdir(ROOT)
    try:
        args = ["build_ext", "--inplace"]
        if not verbose:
            args.insert(0, "-q")
        setup(name="mmltk_b200_native", ext_modules=extensions(debug_bounds),
              cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
              script_args=args)
    finally:
        os.chdir(cwd)
    build_noalloc(verbose)


if __name__ == "__main__":
    if "--host-sanitize" in sys.argv:
        i = sys.argv.index("--host-sanitize")
        print(build_host_selftest(sys.argv[i + 1] if i + 1 < len(sys.argv) else "address,undefined",
                                  verbose="-v" in sys.argv))
    else:
        build(verbose="-v" in sys.argv, debug_bounds="--debug-bounds" in sys.argv)
