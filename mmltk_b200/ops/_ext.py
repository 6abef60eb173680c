"""Loader for the in-tree native extensions.

Two shared objects are built in-tree by ``mmltk_b200.build``:

* ``mmltk_b200/_kernels*.so`` -- the sm_100a CUDA kernels (torch ops);
* ``mmltk_b200/_native*.so``  -- host C++ (LSAP solver, dataset format,
  loader, target packer, COCO evaluator, thread pool).

CUDA tensors never fall back to a PyTorch implementation: if the kernel
extension is missing on a machine with a GPU, ``kernels()`` raises.

``MMLTK_DEBUG_BOUNDS=1`` makes ``kernels()`` load ``_kernels_dbg`` (the same kernels built
with index checks that record an error code in a device status word, read by
``kernels().debug_status()``; ``python -m mmltk_b200.build --debug-bounds``).
"""
from __future__ import annotations

import glob
import importlib
import importlib.util
import os
import sys

_PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_cache = {}


def _load(modname: str):
    if modname in _cache:
        return _cache[modname]
    full = f"mmltk_b200.{modname}"
    mod = None
    err = None
    try:
        import torch  # noqa: F401  (the extension links against libtorch)
        mod = importlib.import_module(full)
    except Exception as e:  # pragma: no cover - reported below
        err = e
    if mod is None:
        cands = glob.glob(os.path.join(_PKG_DIR, f"{modname}.*so"))
        if cands:
            try:
                spec = importlib.util.spec_from_file_location(full, cands[0])
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                sys.modules[full] = mod
            except Exception as e:  # pragma: no cover
                err = e
                mod = None
    _cache[modname] = (mod, err)
    return _cache[modname]


def kernel_module_name() -> str:
    return "_kernels_dbg" if os.environ.get("MMLTK_DEBUG_BOUNDS", "0") == "1" else "_kernels"


def kernels():
    """The CUDA kernel extension; raises if it is not built."""
    mod, err = _load(kernel_module_name())
    if mod is None:
        raise RuntimeError(
            "mmltk_b200 CUDA kernels are not built (run `python -m mmltk_b200.build`); "
            f"import error: {err!r}")
    return mod


def native():
    """The host C++ extension; raises if it is not built."""
    mod, err = _load("_native")
    if mod is None:
        raise RuntimeError(
            "mmltk_b200 native host library is not built (run `python -m mmltk_b200.build`); "
            f"import error: {err!r}")
    return mod


def has_kernels() -> bool:
    return _load(kernel_module_name())[0] is not None


def has_native() -> bool:
    return _load("_native")[0] is not None
