"""ctypes binding to libsabah_rt.so, the sm_100a routed-expert runtime.

Mirrors the reference binding (sabah/runtime/rt.py:1-196): the same QTYPE /
QBLOCK tables, lib(), check(), check_ptr(), row_bytes(), slab helpers and the
same 32 argtype declarations, so code written against the reference module
works unchanged. It additionally declares the v2 MUL_MAT_ID entry point and the
other exports the reference's tests bind by hand, plus this build's extensions
(device-resident banks, synthetic banks).

There is no fallback: if the library is missing, lib() raises
RuntimeUnavailable, and nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))

# ggml type codes (reference rt.py:20-23, plus Q6_K = 14)
QTYPE = {
    "Q5_1": 7, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14,
    "IQ3_XXS": 18, "IQ4_NL": 20, "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "Q2_0": 42,
}
QTYPE_NAME = {v: k for k, v in QTYPE.items()}

# (elements per block, bytes per block) (reference rt.py:26-31, plus Q6_K)
QBLOCK = {
    7: (32, 24), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210),
    18: (256, 98), 20: (32, 18), 21: (256, 110), 22: (256, 82),
    23: (256, 136), 42: (64, 18),
}


class RuntimeUnavailable(Exception):
    """The CUDA runtime library is missing or could not be loaded."""


class SabahCudaError(Exception):
    pass


def library_path() -> str:
    return os.environ.get("SABAH_RT_LIB") or os.path.join(HERE, "libsabah_rt.so")


_lib = None

c_vp, c_sz, c_i, c_f = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_float
c_ull_p = ctypes.POINTER(ctypes.c_ulonglong)

# name -> (argtypes, restype)
SIGNATURES = {
    # the 32 the reference binding declares (rt.py:70-108)
    "sabah_rt_last_error": ([], ctypes.c_char_p),
    "sabah_rt_init": ([c_i], c_i),
    "sabah_rt_shutdown": ([], c_i),
    "sabah_rt_device_count": ([], c_i),
    "sabah_dev_alloc": ([c_sz], c_vp),
    "sabah_dev_free": ([c_vp], None),
    "sabah_host_alloc": ([c_sz], c_vp),
    "sabah_host_free": ([c_vp], None),
    "sabah_dev_mem": ([ctypes.POINTER(c_sz), ctypes.POINTER(c_sz)], c_i),
    "sabah_memcpy_h2d": ([c_vp, c_vp, c_sz], c_i),
    "sabah_memcpy_d2h": ([c_vp, c_vp, c_sz], c_i),
    "sabah_memset_d": ([c_vp, c_i, c_sz], c_i),
    "sabah_h2d_async": ([c_vp, c_vp, c_sz], c_i),
    "sabah_event_create": ([], c_vp),
    "sabah_event_destroy": ([c_vp], None),
    "sabah_event_record_copy": ([c_vp], c_i),
    "sabah_event_record_compute": ([c_vp], c_i),
    "sabah_compute_wait_event": ([c_vp], c_i),
    "sabah_copy_wait_event": ([c_vp], c_i),
    "sabah_event_elapsed_ms": ([c_vp, c_vp], c_f),
    "sabah_event_sync": ([c_vp], c_i),
    "sabah_event_query": ([c_vp], c_i),
    "sabah_sync_copy": ([], c_i),
    "sabah_sync_compute": ([], c_i),
    "sabah_sync_all": ([], c_i),
    "sabah_moe_block": ([c_vp, c_vp, c_vp, c_vp, c_vp, c_i, c_i, c_i, c_i, c_i, c_i, c_i], c_i),
    "sabah_dequant": ([c_vp, c_vp, c_i, c_i, c_i], c_i),
    "sabah_row_bytes": ([c_i, c_i], c_sz),
    "sabah_slab_init": ([c_sz], c_i),
    "sabah_slab_alloc": ([c_sz], c_vp),
    "sabah_slab_free": ([c_vp], None),
    "sabah_slab_destroy": ([], None),
    # the rest of the reference's exports
    "sabah_host_register": ([c_vp, c_sz], c_i),
    "sabah_host_unregister": ([c_vp], c_i),
    "sabah_rt_mul_mat_id_v2": ([c_vp, c_sz, c_sz, c_vp, c_sz, c_i, c_sz, c_vp, c_sz, c_sz, c_i, c_i,
                                c_vp, c_sz, c_sz, c_i, c_i, c_i, c_i, c_vp, c_vp], c_i),
    "sabah_rt_snapshot": ([ctypes.c_char_p, c_sz], c_i),
    "sabah_rt_build_info": ([], ctypes.c_char_p),
    "sabah_rt_host_dequant": ([c_vp, c_vp, c_i, c_i], c_i),
    "sabah_rt_get_diag": ([c_ull_p] * 5, c_i),
    "sabah_rt_get_metrics": ([c_ull_p] * 5, c_i),
    "sabah_rt_resolve_probe": ([c_vp, ctypes.c_char_p, c_sz], c_i),
    "sabah_rt_read_probe": ([ctypes.c_uint64, c_sz, ctypes.c_char_p, c_sz], c_i),
    # extensions of this build
    "sabah_moe_block_ids": ([c_vp, c_vp, c_vp, c_sz, c_sz, c_i, c_vp, c_vp, c_vp, c_vp, c_vp,
                             c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_vp], c_i),
    "sabah_moe_block_ids_noalloc": ([c_vp, c_vp, c_vp, c_sz, c_sz, c_i, c_vp, c_vp, c_vp, c_vp, c_vp,
                                     c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_vp], c_i),
    "sabah_moe_block_gather": ([c_vp, c_vp, c_vp, c_sz, c_sz, c_i, c_vp, c_vp, c_vp, c_vp, c_i, c_vp, c_vp,
                                c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_vp], c_i),
    "sabah_rt_device_error": ([], c_i),
    "sabah_moe_decode": ([c_i, c_vp, c_vp, c_vp, c_sz, c_sz, c_i, c_vp, c_vp, c_vp, c_vp,
                          c_i, c_i, c_i, c_i, c_i, c_i, c_i, c_vp], c_i),
    "sabah_rt_kernel_timing": ([c_i], c_i),
    "sabah_rt_kernel_times": ([ctypes.c_char_p, c_sz], c_i),
    "sabah_synth_rows": ([c_vp, c_i, ctypes.c_longlong, c_i, ctypes.c_ulonglong, c_f, c_vp], c_i),
    "sabah_synth_rows_at": ([c_vp, c_i, ctypes.c_longlong, ctypes.c_longlong, c_i, ctypes.c_ulonglong, c_f, c_vp], c_i),
    "sabah_ep_gather_rows": ([c_vp, c_i, c_vp, c_i, c_i, c_vp, c_vp], c_i),
    "sabah_ep_sum_rows": ([c_vp, c_i, c_vp, c_i, c_i, c_vp, c_vp], c_i),
    "sabah_ep_add": ([c_vp, c_vp, ctypes.c_longlong, c_vp], c_i),
    "sabah_ep_sum_rows_ex": ([c_vp, c_i, c_vp, c_vp, c_i, c_i, c_vp, c_vp, c_i, c_i, c_vp], c_i),
}


def lib():
    """Load the runtime library once, with an actionable error if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    p = library_path()
    if not os.path.exists(p):
        raise RuntimeUnavailable(
            "Sabah CUDA runtime not built: %s\nBuild it with:  python -c "
            "'import __graft_entry__ as g; g.build()'  (or make -C sabah_moe_accelerator_b200/csrc)" % p)
    try:
        L = ctypes.CDLL(p)
    except OSError as e:
        raise RuntimeUnavailable("could not load %s: %s" % (p, e))
    for name, (argt, rest) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.argtypes = argt
        fn.restype = rest
    _lib = L
    return _lib


def last_error() -> str:
    try:
        return (lib().sabah_rt_last_error() or b"").decode("utf-8", "replace")
    except Exception:
        return ""


def check(rc, what="cuda call"):
    if rc is None or (isinstance(rc, int) and rc != 0):
        raise SabahCudaError("%s failed: %s" % (what, last_error()))
    return rc


def check_ptr(p, what="allocation"):
    if not p:
        raise SabahCudaError("%s failed: %s" % (what, last_error()))
    return p


def row_bytes(qt: int, n: int) -> int:
    """Bytes occupied by one row of n elements at quant type qt."""
    be, bb = QBLOCK[qt]
    if n % be:
        raise ValueError("row of %d elements is not a whole number of %s blocks" % (n, QTYPE_NAME.get(qt, qt)))
    return n // be * bb


def available() -> bool:
    try:
        lib()
        return True
    except RuntimeUnavailable:
        return False


def device_count() -> int:
    try:
        return int(lib().sabah_rt_device_count())
    except RuntimeUnavailable:
        return 0


def slab_init(capacity_bytes: int) -> int:
    return check(lib().sabah_slab_init(ctypes.c_size_t(capacity_bytes)), "slab init")


def slab_alloc(bytes_: int) -> int:
    return check_ptr(lib().sabah_slab_alloc(ctypes.c_size_t(bytes_)), "slab alloc")


def slab_free(ptr: int) -> None:
    lib().sabah_slab_free(ctypes.c_void_p(ptr))


def slab_destroy() -> None:
    lib().sabah_slab_destroy()


def host_register(ptr: int, bytes_: int) -> int:
    return check(lib().sabah_host_register(ctypes.c_void_p(ptr), ctypes.c_size_t(bytes_)), "host_register")


def host_unregister(ptr) -> int:
    if isinstance(ptr, ctypes.c_void_p):
        ptr = ptr.value
    return check(lib().sabah_host_unregister(ctypes.c_void_p(ptr)), "host_unregister")


def snapshot() -> dict:
    import json
    buf = ctypes.create_string_buffer(4096)
    lib().sabah_rt_snapshot(buf, 4096)
    return json.loads(buf.value.decode())


def mul_mat_id_v2(source, expert_stride, row_stride, d_x, x_id_stride, x_rows, x_token_stride,
                  d_ids, ids_id_stride, ids_token_stride, n_ids, n_tokens, d_dst, dst_id_stride,
                  dst_token_stride, rows, k, n_experts, qt, stream=None, ids_key=None) -> int:
    """sabah_rt_mul_mat_id_v2 with every pointer given as an int address."""
    return lib().sabah_rt_mul_mat_id_v2(
        c_vp(source), expert_stride, row_stride, c_vp(d_x), x_id_stride, x_rows, x_token_stride,
        c_vp(d_ids), ids_id_stride, ids_token_stride, n_ids, n_tokens, c_vp(d_dst), dst_id_stride,
        dst_token_stride, rows, k, n_experts, qt, c_vp(stream), c_vp(ids_key))
