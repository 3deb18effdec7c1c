"""Hot-tier slab and stream-event plumbing on the GPU, re-hosted from the
reference's model-free smoke tests (tests/test_gpu_smoke.py:55-144)."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MIB = 1 << 20


def test_slab_best_fit_reuses_a_freed_range(gpu_rt):
    from sabah_moe_accelerator_b200 import rt
    a, b, c = rt.slab_alloc(MIB), rt.slab_alloc(MIB), rt.slab_alloc(MIB)
    rt.slab_free(b)
    d = rt.slab_alloc(MIB)
    try:
        assert d == b and d not in (a, c)
    finally:
        for p in (a, c, d):
            rt.slab_free(p)


def test_slab_coalesces_adjacent_frees(gpu_rt):
    from sabah_moe_accelerator_b200 import rt
    a, b, c = rt.slab_alloc(MIB), rt.slab_alloc(MIB), rt.slab_alloc(MIB)
    for p in (a, b, c):
        rt.slab_free(p)
    big = rt.slab_alloc(3 * MIB)
    try:
        assert big == a
    finally:
        rt.slab_free(big)


def test_slab_returns_null_when_no_range_fits(gpu_rt):
    assert not gpu_rt.sabah_slab_alloc(ctypes.c_size_t(1 << 62))


def test_slab_destroy_and_reinit(gpu_rt):
    from sabah_moe_accelerator_b200 import rt
    cap = int(os.environ.get("SABAH_LLAMA_HOT_BYTES") or 0) or (2 << 30)
    gpu_rt.sabah_slab_destroy()
    try:
        rt.slab_init(4 * MIB)
        p = rt.slab_alloc(MIB)
        assert p
        rt.slab_free(p)
        assert not gpu_rt.sabah_slab_alloc(ctypes.c_size_t(8 * MIB))
    finally:
        gpu_rt.sabah_slab_destroy()
        rt.slab_init(cap)


def test_copy_wait_event_contract(gpu_rt):
    from sabah_moe_accelerator_b200 import rt
    L = gpu_rt
    n = 4096
    src = np.arange(n, dtype=np.uint8)
    d = rt.check_ptr(L.sabah_dev_alloc(n), "dev alloc")
    host = rt.check_ptr(L.sabah_host_alloc(n), "host alloc")
    ev = rt.check_ptr(L.sabah_event_create(), "event")
    try:
        rt.check(L.sabah_event_record_compute(ev), "record")
        rt.check(L.sabah_copy_wait_event(ev), "copy wait")
        rt.check(L.sabah_h2d_async(d, src.ctypes.data, n), "h2d async")
        rt.check(L.sabah_sync_all(), "sync")
        assert L.sabah_event_query(ev) == 1
        rt.check(L.sabah_memcpy_d2h(host, d, n), "d2h")
        got = np.ctypeslib.as_array(ctypes.cast(host, ctypes.POINTER(ctypes.c_uint8)), (n,))
        assert np.array_equal(got, src)
    finally:
        L.sabah_event_destroy(ev)
        L.sabah_host_free(host)
        L.sabah_dev_free(d)


def test_pinned_pool_reuses_blocks(gpu_rt):
    L = gpu_rt
    a = L.sabah_host_alloc(1 << 22)
    L.sabah_host_free(a)
    b = L.sabah_host_alloc(1 << 22)     # the freed 4 MiB block is handed out again
    assert a == b
    c = L.sabah_host_alloc(1 << 22)     # while b is live, a second request gets a new block
    assert c != b
    L.sabah_host_free(b)
    L.sabah_host_free(c)


def test_dev_mem_reports_a_b200_sized_device(gpu_rt):
    f, t = ctypes.c_size_t(), ctypes.c_size_t()
    assert gpu_rt.sabah_dev_mem(ctypes.byref(f), ctypes.byref(t)) == 0
    assert t.value > (100 << 30) and 0 < f.value <= t.value
