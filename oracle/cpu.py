"""ctypes wrapper of the CPU oracle (oracle/sabah_oracle.c) and of the reference
build under oracle/_ref/.

TEST INFRASTRUCTURE. Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg import this module, as the checker or as the timed CPU baseline.
The product never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libsabah_rt_ref.so")

QBLOCK = {
    7: (32, 24), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210),
    18: (256, 98), 20: (32, 18), 21: (256, 110), 22: (256, 82),
    23: (256, 136), 42: (64, 18),
}

_lib = None
_ref = None

c_vp, c_sz, c_i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_dequant.argtypes = [c_vp, c_vp, c_i, ctypes.c_int64]
        L.orc_mmid_f64.argtypes = [c_vp, c_sz, c_sz, c_vp, c_sz, c_i, c_sz, c_vp, c_sz, c_sz, c_i, c_i,
                                   c_vp, c_i, c_i, c_i, c_i]
        L.orc_moe_block_f64.argtypes = [c_vp, c_vp, c_vp, c_vp, c_vp, c_vp, c_i, c_i, c_i, c_i, c_i, c_i, c_vp]
        L.orc_decode_f32.argtypes = [c_vp, c_vp, c_vp, c_sz, c_sz, c_i, c_i, c_i, c_vp, c_vp, c_vp,
                                     c_i, c_i, c_i, c_i, c_vp]
        _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref_lib():
    """The reference runtime compiled from its own sources (oracle/build_ref.sh)."""
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_PATH)
        L.sabah_rt_host_dequant.argtypes = [c_vp, c_vp, c_i, c_i]
        L.sabah_rt_host_dequant.restype = c_i
        _ref = L
    return _ref


def row_bytes(qt: int, n: int) -> int:
    be, bb = QBLOCK[qt]
    assert n % be == 0
    return n // be * bb


def dequant(raw: np.ndarray, qt: int, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n, np.float32)
    rc = lib().orc_dequant(raw.ctypes.data, out.ctypes.data, qt, n)
    if rc != 0:
        raise ValueError("oracle cannot dequantize type %d" % qt)
    return out


def ref_dequant(raw: np.ndarray, qt: int, n: int):
    """The reference's own host dequantizer, or None if it lacks the type."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n, np.float32)
    return out if ref_lib().sabah_rt_host_dequant(raw.ctypes.data, out.ctypes.data, qt, n) == 0 else None


def mmid_f64(source: np.ndarray, expert_stride: int, row_stride: int, x: np.ndarray, x_rows: int,
             ids: np.ndarray, rows: int, k: int, n_experts: int, qt: int) -> np.ndarray:
    """fp64 MUL_MAT_ID over dense inputs: x [T][x_rows][k] fp32, ids [T][n_ids] i32.
    Returns [T][n_ids][rows] float64."""
    source = np.ascontiguousarray(source, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    T, n_ids = ids.shape
    out = np.empty((T, n_ids, rows), np.float64)
    rc = lib().orc_mmid_f64(source.ctypes.data, expert_stride, row_stride, x.ctypes.data, k * 4, x_rows,
                            x_rows * k * 4, ids.ctypes.data, 4, n_ids * 4, n_ids, T, out.ctypes.data,
                            rows, k, n_experts, qt)
    if rc != 0:
        raise ValueError("oracle mmid failed (%d)" % rc)
    return out


def moe_block_f64(gate: np.ndarray, up: np.ndarray, down: np.ndarray, ids, w, x: np.ndarray,
                  d_model: int, ff: int, qt_gate: int, qt_up: int, qt_down: int, with_h: bool = False):
    """fp64 reference_block for one token; gate/up/down are whole banks
    [n_experts][rows][row bytes] as uint8 arrays."""
    gate = np.ascontiguousarray(gate, dtype=np.uint8)
    up = np.ascontiguousarray(up, dtype=np.uint8)
    down = np.ascontiguousarray(down, dtype=np.uint8)
    n = len(ids)
    gs = row_bytes(qt_gate, d_model) * ff
    us = row_bytes(qt_up, d_model) * ff
    ds = row_bytes(qt_down, ff) * d_model
    gp = (c_vp * n)(*[gate.ctypes.data + int(e) * gs for e in ids])
    up_ = (c_vp * n)(*[up.ctypes.data + int(e) * us for e in ids])
    dp = (c_vp * n)(*[down.ctypes.data + int(e) * ds for e in ids])
    w = np.ascontiguousarray(w, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(d_model, np.float64)
    h = np.empty((n, ff), np.float64) if with_h else None
    rc = lib().orc_moe_block_f64(gp, up_, dp, w.ctypes.data, x.ctypes.data, out.ctypes.data, d_model, ff, n,
                                 qt_gate, qt_up, qt_down, h.ctypes.data if with_h else None)
    if rc != 0:
        raise ValueError("oracle block failed")
    return (out, h) if with_h else out


def decode_f32(gate_bases, up_bases, down_bases, gu_expert_stride: int, d_expert_stride: int, qt_gu: int,
               qt_d: int, ids: np.ndarray, w: np.ndarray, x: np.ndarray, d_model: int, ff: int,
               n_threads: int, use_reference_dequant: bool = False) -> np.ndarray:
    """fp32 multi-layer decode (the timed CPU baseline). *_bases are host
    addresses of each layer's expert bank; ids/w are [L][n_used]. Returns the
    final x (x_{L+1} = x_L + y_L)."""
    L = len(gate_bases)
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    xx = np.array(x, dtype=np.float32, copy=True)
    dq = None
    if use_reference_dequant:
        dq = ctypes.cast(ref_lib().sabah_rt_host_dequant, c_vp)
    rc = lib().orc_decode_f32((c_vp * L)(*gate_bases), (c_vp * L)(*up_bases), (c_vp * L)(*down_bases),
                              gu_expert_stride, d_expert_stride, qt_gu, qt_d, L, ids.ctypes.data,
                              w.ctypes.data, xx.ctypes.data, d_model, ff, ids.shape[1], n_threads, dq)
    if rc != 0:
        raise ValueError("oracle decode failed")
    return xx


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    n = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / n) if n > 0 else float(np.linalg.norm(a - b))
