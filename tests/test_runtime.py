"""Host runtime: CPU sets, per-rank shards, worker budgets, thread split, pinning and
priority (the native exec_policy module and mmltk_b200.utils.runtime)."""
import json
import os
import subprocess
import sys

import pytest

from mmltk_b200.ops._ext import native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shards_are_contiguous_and_cover_the_set():
    n = native()
    cpus = list(range(3, 13))
    shards = [list(n.shard_cpus(cpus, r, 3)) for r in range(3)]
    assert shards == [[3, 4, 5, 6], [7, 8, 9], [10, 11, 12]]
    assert sum(shards, []) == cpus
    assert list(n.shard_cpus([0, 1], 0, 3)) == []          # fewer CPUs than ranks
    with pytest.raises(ValueError):
        n.shard_cpus(cpus, 3, 3)


def test_worker_budget_clamp():
    n = native()
    assert n.clamp_workers(0, 8, 0, 3) == 8        # 0: one per CPU
    assert n.clamp_workers(32, 8, 0, 3) == 8       # never above the CPU count
    assert n.clamp_workers(2, 8, 0, 3) == 3        # never below the minimum
    assert n.clamp_workers(6, 8, 4, 1) == 4        # reserved CPUs are not handed out


def test_runtime_split():
    n = native()
    assert n.split_runtime(8, 1, 2) == {"loader": 3, "gather": 2, "lane": 1, "cpu": 4}
    assert n.split_runtime(2, 1, 2) == {"loader": 1, "gather": 1, "lane": 1, "cpu": 1}
    # lanes and loader are clamped so the CPU pool keeps one thread
    assert n.split_runtime(3, 4, 2) == {"loader": 1, "gather": 1, "lane": 1, "cpu": 1}
    assert n.split_runtime(6, 2, 0) == {"loader": 0, "gather": 0, "lane": 2, "cpu": 4}
    for w in range(3, 40):
        s = n.split_runtime(w, 2, 3)
        assert s["loader"] + s["lane"] + s["cpu"] == w and s["cpu"] >= 1


def test_cpu_affinity_resolution():
    n = native()
    allowed = list(n.allowed_cpus())
    assert list(n.resolve_cpu_affinity("")) == allowed
    assert list(n.resolve_cpu_affinity(str(allowed[0]))) == [allowed[0]]
    with pytest.raises(ValueError):
        n.resolve_cpu_affinity("100000")                   # outside the allowed set
    assert list(n.cpu_slice([4, 5, 6], 2, 3)) == [4, 5, 6]  # wraps, sorted, unique


_CHILD = r"""
import json, os, sys
sys.path.insert(0, sys.argv[1])
import torch
from mmltk_b200.utils.runtime import setup_host_runtime
rt = setup_host_runtime(workers=0, lanes=1, prefetch=2, cpu_affinity="", pin=True, high_priority=True)
print(json.dumps({"main": rt.main_cpus, "now": sorted(os.sched_getaffinity(0)), "loader": rt.loader_cpus,
                  "split": rt.split, "workers": rt.workers, "nice": rt.policy["nice"], "cpus": rt.cpus,
                  "pool_threads": rt.pool_threads}))
"""


def test_setup_host_runtime_pins_the_lane_thread():
    # in a child: pinning and the global pool must not leak into this test process
    out = subprocess.run([sys.executable, "-c", _CHILD, ROOT], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    r = json.loads(out.stdout.strip().splitlines()[-1])
    assert r["now"] == r["main"]
    if len(r["cpus"]) >= 3:
        assert r["loader"][0] not in r["main"]              # the producer's CPU is left to the loader
    assert r["workers"] == max(3, len(r["cpus"]))
    s = r["split"]
    assert s["loader"] + s["lane"] + s["cpu"] == r["workers"]
    assert r["nice"] <= 0                                  # never raised; lowered where permitted


def test_rank_plan_shards_cpus_and_workers():
    from mmltk_b200.parallel.launch import rank_plan
    n = native()
    allowed = list(n.allowed_cpus())
    plan = rank_plan(2, 8, "")
    assert len(plan) == 2
    joined = []
    for _per, cpus in plan:
        if cpus:
            joined += list(n.parse_cpuset(cpus))
    if len(allowed) >= 2:
        assert joined == allowed


def test_loader_accepts_cpu_placement(tmp_path):
    from mmltk_b200.data.compiler import compile_split
    from mmltk_b200.data.loader import BatchLoader
    from mmltk_b200.data.source import write_synthetic_source
    write_synthetic_source(str(tmp_path / "src"), splits=("train",), images=4, size=(32, 32))
    path = compile_split(str(tmp_path / "src"), str(tmp_path / "bin"), "train", 32, 32)["path"]
    cpu0 = int(native().allowed_cpus()[0])
    bl = BatchLoader(path, 2, shuffle=False, pixels="uint8", max_targets=4, cpus=[cpu0])
    got = [idx for _img, _t, idx in bl]
    assert sorted(sum(got, [])) == [0, 1, 2, 3]


def test_host_selftest_under_asan_ubsan():
    """The torch-free host runtime (LSAP, worker pool, PNG codec, resizers) built with
    AddressSanitizer + UndefinedBehaviorSanitizer and run: any invalid access or UB aborts it."""
    import shutil
    import subprocess
    if shutil.which("g++") is None:
        pytest.skip("no host compiler")
    from mmltk_b200.build import build_host_selftest
    exe = build_host_selftest("address,undefined")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "host selftest ok" in r.stdout, r.stdout + r.stderr
