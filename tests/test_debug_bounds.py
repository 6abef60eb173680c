"""Debug bounds-check build (`_kernels_dbg`, MMLTK_DEBUG_BOUNDS=1): data-dependent indices that are
out of range are reported through a device status word instead of trapping, and the kernels keep
their release behaviour (the index is clamped or the element skipped), so the bad input is never
dereferenced.  The GPU case runs in a fresh process that loads only the debug build."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import torch
from mmltk_b200.ops import kernels
k = kernels()
assert k.debug_build(), "expected the debug-bounds build"
dev = torch.device("cuda", 0)
B, Q, C, T = 2, 40, 91, 6
logits = torch.randn(B, Q, C, device=dev).bfloat16()
boxes = (torch.rand(B, Q, 4, device=dev) * 0.5 + 0.25).bfloat16()
tb = torch.rand(B, T, 4, device=dev) * 0.4 + 0.3
counts = torch.tensor([3, 5], dtype=torch.int32, device=dev)
labels = torch.randint(0, C, (B, T), device=dev)
ok = k.matcher_cost([logits], [boxes], labels, tb, counts, 2.0, 5.0, 2.0, 0.25)
assert k.debug_status() == 0, "in-range inputs must not report"
labels[1, 2] = C + 4                     # an out-of-range class id, set on the host side
bad = k.matcher_cost([logits], [boxes], labels, tb, counts, 2.0, 5.0, 2.0, 0.25)
code = k.debug_status()
assert code == 0x101, hex(code)
assert k.debug_status() == 0, "the status word is cleared by the read"
assert torch.isfinite(bad).all()
counts[0] = T + 3                        # more targets than slots
k.matcher_cost([logits], [boxes], labels.clamp(max=C - 1), tb, counts, 2.0, 5.0, 2.0, 0.25)
assert k.debug_status() == 0x102
print("debug-bounds ok")
"""


def _dbg_built():
    import glob
    return bool(glob.glob(os.path.join(ROOT, "mmltk_b200", "_kernels_dbg.*so")))


@pytest.mark.gpu
def test_debug_build_reports_out_of_range_indices(cuda_device):
    if not _dbg_built():
        from mmltk_b200.build import build
        build(debug_bounds=True)
    env = dict(os.environ, MMLTK_DEBUG_BOUNDS="1", PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-c", SCRIPT], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "debug-bounds ok" in r.stdout, r.stdout + r.stderr


def test_release_loader_ignores_debug_variant(monkeypatch):
    """Without MMLTK_DEBUG_BOUNDS the loader names the release module; with it, the debug one."""
    from mmltk_b200.ops import _ext
    monkeypatch.delenv("MMLTK_DEBUG_BOUNDS", raising=False)
    assert _ext.kernel_module_name() == "_kernels"
    monkeypatch.setenv("MMLTK_DEBUG_BOUNDS", "1")
    assert _ext.kernel_module_name() == "_kernels_dbg"
