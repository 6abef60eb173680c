#!/usr/bin/env python3
"""Build the reference arm of ``bench.py``: rlewkowicz/mmltk's own libtorch sources, unmodified.

The reference is a CMake / libtorch C++20 project without Python packaging, so
``pip install --target baseline/_ref <reference>`` cannot install it ("Neither 'setup.py' nor
'pyproject.toml' found").  Its full CMake graph cannot be configured here either: the dataset
compiler / loader sources it lists (``src/dataset/**``) are absent from the snapshot, and it requires
ONNX, ONNX Runtime and TensorRT.  The model, loss, matcher, optimizer, MSDeformAttn and post-process
code does not need any of those, so this script:

1. copies the reference's ``src/``, ``include/`` and the vendored ``third_party/spdlog`` and
   ``third_party/json`` trees, byte for byte, into ``baseline/_ref/reference`` (so the arm runs from
   ``baseline/_ref`` on a machine where the reference checkout is absent);
2. compiles the translation units of the reference's ``mmltk_rfdetr_cuda_ops``, ``mmltk_rfdetr_torch``
   and ``mmltk_core`` targets that the training / inference step reaches, with the reference's
   Release settings (``-O3 -DNDEBUG``, ``MMLTK_ENABLE_PROFILING=0``, C++20, CUDA for sm_100 as in
   its ``MMLTK_CUDA_ARCHITECTURES`` list), plus ``ref_harness.cpp`` (which only calls the reference's
   public API), into ``baseline/_ref/mmltk_ref*.so`` with ``torch.utils.cpp_extension``;
3. adds link shims for code the benchmark never reaches: ``shim/onnx/onnx_pb.h`` (a forward
   declaration of ``ModelProto``) and ``shim/onnx_io_stub.cpp`` (the ONNX file writer, which throws)
   because the ONNX protobuf library is not in this image and only ``export_onnx`` uses it; and
   ``shim/dataset_loader_stub.cpp`` (the two ``DatasetLoader`` methods ``LoaderBatchGuard`` names,
   which throw) because the loader's sources are missing from the reference snapshot.

Usage: ``python baseline/build_reference.py [--src <reference checkout>] [--jobs N]``.
"""
from __future__ import annotations

import argparse
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
COPY = os.path.join(OUT, "reference")

# translation units reached by NativeRfDetrModel forward/backward, detection_loss_dict,
# NativeAdamW / ModelEma, MSDeformAttn and post-processing (reference-relative paths)
SOURCES = [
    "src/rfdetr/layers/model.cpp",
    "src/rfdetr/layers/modules.cpp",
    "src/rfdetr/layers/model_components.cpp",
    "src/rfdetr/layers/model_config.cpp",
    "src/rfdetr/layers/ms_deform_attn_op.cpp",
    "src/rfdetr/layers/ms_deform_attn_cuda_wrapper.cpp",
    "src/rfdetr/layers/training_mask_ops_cuda_wrapper.cpp",
    "src/rfdetr/layers/mask_pack_cuda_wrapper.cpp",
    "src/rfdetr/cuda/ms_deform_attn_cuda.cu",
    "src/rfdetr/cuda/training_mask_ops_cuda.cu",
    "src/rfdetr/cuda/mask_pack_cuda.cu",
    "src/rfdetr/cuda/detr_ops_cuda.cu",
    "src/rfdetr/detection_ops.cpp",
    "src/rfdetr/checkpoint.cpp",
    "src/rfdetr/checkpoint/python_checkpoint_bridge.cpp",
    "src/rfdetr/weight_catalog.cpp",
    "src/rfdetr/onnx_lowering.cpp",
    "src/rfdetr/training/native_optimizer.cpp",
    "src/rfdetr/utils/scipy_rectangular_lsap.cpp",
    "src/rfdetr/inference/postprocess.cpp",
    "src/rfdetr/gpu_augment.cpp",
    "src/rfdetr/cuda/gpu_augment_cuda.cu",
    "src/rfdetr/target_builder.cpp",
    "src/mmltk_logging.cpp",
    "src/profile_utils.cpp",
    "src/worker_pool.cpp",
    "src/cpu_affinity.cpp",
    "src/execution_policy.cpp",
]

COPY_TREES = ["src", "include", "third_party/spdlog", "third_party/json", "LICENSE", "NOTICE"]


def copy_reference(src_root: str) -> None:
    """Byte-for-byte copy of the trees the build reads (skips the GUI / browser trees)."""
    skip = {os.path.join("src", "gui"), os.path.join("src", "browser")}
    for rel in COPY_TREES:
        s = os.path.join(src_root, rel)
        d = os.path.join(COPY, rel)
        if os.path.isfile(s):
            os.makedirs(os.path.dirname(d), exist_ok=True)
            shutil.copy2(s, d)
            continue
        for root, dirs, files in os.walk(s):
            relroot = os.path.relpath(root, src_root)
            if any(relroot == k or relroot.startswith(k + os.sep) for k in skip):
                dirs[:] = []
                continue
            os.makedirs(os.path.join(COPY, relroot), exist_ok=True)
            for f in files:
                shutil.copy2(os.path.join(root, f), os.path.join(COPY, relroot, f))
    # model.cpp includes one header of the GUI tree (subprocess helpers for the ONNX simplifier)
    for rel in ("src/gui/subprocess_utils.h", "src/gui/console_output.h"):
        s = os.path.join(src_root, rel)
        if os.path.exists(s):
            os.makedirs(os.path.dirname(os.path.join(COPY, rel)), exist_ok=True)
            shutil.copy2(s, os.path.join(COPY, rel))


def build(jobs: int, verbose: bool) -> str:
    os.environ.setdefault("MAX_JOBS", str(jobs))
    from torch.utils.cpp_extension import load

    inc = [os.path.join(HERE, "shim"), os.path.join(COPY, "include"), os.path.join(COPY, "src"),
           os.path.join(COPY, "third_party", "spdlog", "include"), os.path.join(COPY, "third_party", "json", "include"),
           os.path.join(COPY, "third_party"), "/usr/local/cuda/include"]
    defs = ["-DMMLTK_ENABLE_PROFILING=0", '-DMMLTK_BUILD_CONFIG=\\"Release\\"', "-DNDEBUG"]
    srcs = [os.path.join(COPY, s) for s in SOURCES]
    srcs += [os.path.join(HERE, "shim", "onnx_io_stub.cpp"), os.path.join(HERE, "shim", "dataset_loader_stub.cpp"),
             os.path.join(HERE, "ref_harness.cpp")]
    build_dir = os.path.join(OUT, "build")
    os.makedirs(build_dir, exist_ok=True)
    load(name="mmltk_ref", sources=srcs, extra_include_paths=inc,
         extra_cflags=["-O3", "-std=c++20", "-w"] + defs,
         extra_cuda_cflags=["-O3", "-std=c++20", "-w", "--expt-relaxed-constexpr", "--extended-lambda",
                            "-gencode", "arch=compute_100,code=sm_100"] + defs,
         extra_ldflags=["-lcudart", "-lcuda"],
         build_directory=build_dir, verbose=verbose, with_cuda=True, is_python_module=True)
    so = [f for f in os.listdir(build_dir) if f.startswith("mmltk_ref") and f.endswith(".so")]
    if not so:
        raise RuntimeError("reference build produced no module")
    shutil.copy2(os.path.join(build_dir, so[0]), os.path.join(OUT, so[0]))
    return os.path.join(OUT, so[0])


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=os.environ.get("MMLTK_REFERENCE_SRC", "/root/reference"))
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--no-copy", action="store_true", help="reuse baseline/_ref/reference")
    args = ap.parse_args()
    os.makedirs(OUT, exist_ok=True)
    if not args.no_copy:
        if not os.path.isdir(os.path.join(args.src, "src", "rfdetr")):
            print(f"reference sources not found at {args.src}", file=sys.stderr)
            return 2
        copy_reference(args.src)
    path = build(args.jobs, args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
