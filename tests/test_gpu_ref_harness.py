"""The drop-in claim, tested by the reference's own caller code: its model-free
GPU test (tests/test_gpu_smoke.py of the reference project: the device slab,
sabah_copy_wait_event, and a HotTier over a fake bank), with its own
sabah/runtime/rt.py and hot_tier.py, unmodified, loading THIS build's
libsabah_rt.so through SABAH_RT_LIB (the reference binding's own switch,
sabah/runtime/rt.py:46-47). __graft_entry__.build() copies those files from the
reference into the git-ignored baseline/_ref/harness.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys

import pytest

from conftest import LIB, ROOT

pytestmark = pytest.mark.gpu

HARNESS = os.path.join(ROOT, "baseline", "_ref", "harness")


def test_reference_gpu_smoke_passes_on_this_library():
    test = os.path.join(HARNESS, "tests", "test_gpu_smoke.py")
    assert os.path.exists(test), "reference harness not staged (python __graft_entry__.py build): " + test
    env = dict(os.environ, SABAH_RT_LIB=LIB, PYTHONPATH=HARNESS)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", test], cwd=HARNESS, env=env,
                       capture_output=True, text=True, timeout=900)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    m = re.search(r"(\d+) passed", out)
    assert m and int(m.group(1)) >= 8, out[-2000:]
    assert "skipped" not in out and "failed" not in out, out[-2000:]
