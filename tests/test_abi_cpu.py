"""The drop-in boundary, checked without a GPU.

  * libsabah_rt.so loads and exports every symbol include/sabah_rt.h declares,
    and every symbol the reference runtime exports (the 42 of
    sabah/runtime/cuda/sabah_rt.cu:3039-3903);
  * the host-side entry points behave as the reference's do: build info,
    row bytes, host dequant (bit-exact with gguf-py and the oracle), and the
    -1 + last_error convention when the runtime is not initialised.
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "sabah_rt.h")

# the reference runtime's exports (nm -D of its Linux build)
REFERENCE_EXPORTS = """
sabah_compute_wait_event sabah_copy_wait_event sabah_dequant sabah_dev_alloc sabah_dev_free sabah_dev_mem
sabah_event_create sabah_event_destroy sabah_event_elapsed_ms sabah_event_query sabah_event_record_compute
sabah_event_record_copy sabah_event_sync sabah_h2d_async sabah_host_alloc sabah_host_free sabah_host_register
sabah_host_unregister sabah_memcpy_d2h sabah_memcpy_h2d sabah_memset_d sabah_moe_block sabah_row_bytes
sabah_rt_build_info sabah_rt_device_count sabah_rt_get_diag sabah_rt_get_metrics sabah_rt_host_dequant
sabah_rt_init sabah_rt_last_error sabah_rt_mul_mat_id_v2 sabah_rt_read_probe sabah_rt_resolve_probe
sabah_rt_shutdown sabah_rt_snapshot sabah_slab_alloc sabah_slab_destroy sabah_slab_free sabah_slab_init
sabah_sync_all sabah_sync_compute sabah_sync_copy
""".split()

TYPES = {"Q5_1": 7, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ3_XXS": 18, "IQ4_NL": 20,
         "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "Q2_0": 42}


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sabah_\w+)\s*\(", text)))


def _exported():
    from conftest import LIB
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def test_reference_has_42_exports():
    assert len(REFERENCE_EXPORTS) == 42


def test_every_declared_symbol_is_exported(rtlib):
    exported = _exported()
    declared = _declared()
    assert len(declared) >= 45
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    for s in declared:
        assert hasattr(rtlib, s)


def test_every_reference_export_is_declared_and_exported(rtlib):
    declared, exported = set(_declared()), _exported()
    assert not [s for s in REFERENCE_EXPORTS if s not in declared]
    assert not [s for s in REFERENCE_EXPORTS if s not in exported]


def test_no_stray_exports(rtlib):
    stray = [s for s in _exported() if not s.startswith("sabah_")]
    assert not stray, stray


def test_rt_binding_covers_every_export(rtlib):
    from sabah_moe_accelerator_b200 import rt
    assert set(_declared()) == set(rt.SIGNATURES)


def test_build_info(rtlib):
    assert rtlib.sabah_rt_build_info().decode() == "sabah_rt abi=v2 sentinel=0"


@pytest.mark.parametrize("name", sorted(TYPES))
def test_row_bytes(rtlib, name):
    from sabah_moe_accelerator_b200 import rt
    qt = TYPES[name]
    be, bb = rt.QBLOCK[qt]
    assert rtlib.sabah_row_bytes(qt, 2048) == 2048 // be * bb == rt.row_bytes(qt, 2048)
    assert rtlib.sabah_row_bytes(qt, be + 0) == bb
    assert rtlib.sabah_row_bytes(99, 256) == 0
    if be > 32:
        assert rtlib.sabah_row_bytes(qt, 32) == 0


@pytest.mark.parametrize("name", sorted(TYPES))
def test_host_dequant_bit_exact(rtlib, orc, golden, name):
    """sabah_rt_host_dequant == oracle == gguf-py / reference, bit for bit."""
    qt = TYPES[name]
    raw = np.ascontiguousarray(golden["raw_" + name])
    n = raw.shape[0] * orc.QBLOCK[qt][0]
    got = np.empty(n, np.float32)
    assert rtlib.sabah_rt_host_dequant(raw.ctypes.data, got.ctypes.data, qt, n) == 0
    assert np.array_equal(got.view(np.uint32), orc.dequant(raw, qt, n).view(np.uint32))
    for side in ("gguf_", "ref_"):
        if side + name in golden:
            assert np.array_equal(got.view(np.uint32), golden[side + name].view(np.uint32))


def test_host_dequant_rejects_bad_geometry(rtlib):
    raw = np.zeros(220, np.uint8)
    out = np.empty(512, np.float32)
    assert rtlib.sabah_rt_host_dequant(raw.ctypes.data, out.ctypes.data, 21, 100) == -1
    assert rtlib.sabah_rt_host_dequant(raw.ctypes.data, out.ctypes.data, 5, 256) == -1


def test_v2_without_init_fails_with_message(rtlib):
    from sabah_moe_accelerator_b200 import rt
    x = np.zeros(64, np.float32)
    rc = rt.mul_mat_id_v2(x.ctypes.data, 1, 1, x.ctypes.data, 4, 1, 4, x.ctypes.data, 4, 4, 1, 1,
                          x.ctypes.data, 4, 4, 1, 32, 1, 8)
    assert rc == -1
    assert "invalid" in rt.last_error()


def test_device_count_is_safe_without_gpu(rtlib):
    from sabah_moe_accelerator_b200 import rt
    assert rt.device_count() >= 0


def test_resolve_probe_names_a_mapped_file(rtlib, tmp_path):
    import mmap
    p = tmp_path / "blob.bin"
    data = bytes(range(256)) * 64
    p.write_bytes(data)
    with open(p, "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        arr = np.frombuffer(mm, dtype=np.uint8)
        buf = ctypes.create_string_buffer(1024)
        assert rtlib.sabah_rt_resolve_probe(ctypes.c_void_p(arr.ctypes.data + 4096 + 17), buf, 1024) == 0
        msg = buf.value.decode()
        assert "resolved=1" in msg and str(p) in msg and "offset=4113" in msg
        assert rtlib.sabah_rt_read_probe(4113, 8, buf, 1024) == 0
        assert buf.value.decode().endswith("first8=11 12 13 14 15 16 17 18 ")
        del arr
        mm.close()
    heap = np.zeros(16, np.uint8)
    assert rtlib.sabah_rt_resolve_probe(ctypes.c_void_p(heap.ctypes.data), buf, 1024) == -1
    assert buf.value.decode().startswith("resolved=0")
