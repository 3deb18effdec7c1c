"""Shared fixtures. Tests marked `gpu` need a B200; everything else runs on CPU.

The product library (sabah_moe_accelerator_b200/libsabah_rt.so) and the CPU
oracle (oracle/_build/liboracle.so) are built on first use if absent.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG = os.path.join(ROOT, "sabah_moe_accelerator_b200")
LIB = os.path.join(PKG, "libsabah_rt.so")
GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _ensure_built():
    if not os.path.exists(LIB):
        subprocess.run(["make", "-s", "-C", os.path.join(PKG, "csrc")], check=True)


@pytest.fixture(scope="session")
def rtlib():
    _ensure_built()
    from sabah_moe_accelerator_b200 import rt
    return rt.lib()


@pytest.fixture(scope="session")
def orc():
    from oracle import cpu
    cpu.lib()
    return cpu


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


@pytest.fixture(scope="session")
def gpu_rt(rtlib):
    """Initialised runtime on device 0 (gpu tests only)."""
    from sabah_moe_accelerator_b200 import rt
    if rt.device_count() < 1:
        pytest.fail("gpu test collected but no CUDA device is visible")
    rt.check(rtlib.sabah_rt_init(0), "rt_init")
    yield rtlib
