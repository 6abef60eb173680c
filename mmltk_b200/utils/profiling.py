"""Lightweight profiling: NVTX ranges and host-side counters.

Counterpart of the reference's ``MMLTK_PROFILE_SCOPE / ADD / SET`` macros and
its report (`include/profile_utils.h:5-126`, `src/profile_utils.cpp`).  With
``MMLTK_PROFILE=1`` scopes accumulate call counts and wall durations, ``add`` /
``set`` record counters, and at exit the totals are appended as one JSON line
to ``MMLTK_PROFILE_LOG`` (default ``mmltk_profile.jsonl``).  NVTX ranges are
always emitted on CUDA so external timelines show the phases; they cost a few
hundred nanoseconds each.
"""
from __future__ import annotations

import atexit
import contextlib
import json
import os
import threading
import time
from collections import defaultdict
from typing import Dict

import torch

__all__ = ["enabled", "scope", "add", "set_value", "report", "reset", "flush"]

enabled = os.environ.get("MMLTK_PROFILE", "") not in ("", "0", "false", "False")
_lock = threading.Lock()
_durations: Dict[str, float] = defaultdict(float)
_calls: Dict[str, int] = defaultdict(int)
_counters: Dict[str, float] = defaultdict(float)
_values: Dict[str, float] = {}
_nvtx = torch.cuda.is_available()


@contextlib.contextmanager
def scope(name: str):
    if _nvtx:
        torch.cuda.nvtx.range_push(name)
    t0 = time.perf_counter() if enabled else 0.0
    try:
        yield
    finally:
        if enabled:
            dt = time.perf_counter() - t0
            with _lock:
                _durations[name] += dt
                _calls[name] += 1
        if _nvtx:
            torch.cuda.nvtx.range_pop()


def add(name: str, value: float = 1.0) -> None:
    if enabled:
        with _lock:
            _counters[name] += value


def set_value(name: str, value: float) -> None:
    if enabled:
        with _lock:
            _values[name] = value


def report() -> dict:
    with _lock:
        return {"scopes": {k: {"calls": _calls[k], "seconds": _durations[k]} for k in sorted(_durations)},
                "counters": dict(sorted(_counters.items())), "values": dict(sorted(_values.items()))}


def reset() -> None:
    with _lock:
        _durations.clear()
        _calls.clear()
        _counters.clear()
        _values.clear()


def flush(path: str = "") -> None:
    if not enabled:
        return
    path = path or os.environ.get("MMLTK_PROFILE_LOG", "mmltk_profile.jsonl")
    rec = {"event": "mmltk.profile", "pid": os.getpid(), "time": time.time(), **report()}
    with open(path, "a") as f:
        f.write(json.dumps(rec) + "\n")


if enabled:
    atexit.register(flush)
