"""Child process that runs the REFERENCE runtime, oracle/_ref/libsabah_rt_ref.so
(sabah/runtime/cuda/sabah_rt.cu compiled unmodified by oracle/build_ref.sh),
on inputs from an .npz file, and saves its outputs. Nothing of this
repository's library is loaded here. Test infrastructure only.

  python tests/ref_child.py mmid  IN.npz OUT.npz REPS
      sabah_rt_mul_mat_id_v2 (sabah_rt.cu:3494-3833) with a HOST source, the
      llama.cpp contract: `source` [E][rows][row bytes], x [T][x_rows][k], ids
      [T][n_ids]; REPS + 1 identical calls (the first fills the hot tier).
  python tests/ref_child.py block IN.npz OUT.npz REPS
      sabah_moe_block (sabah_rt.cu:3362-3378) over device banks and a device
      pointer table [gate x n, up x n, down x n], as the harness's executor
      builds it (sabah/runtime/executor.py:61-99).

With SABAH_LLAMA_EVENTS=1 and SABAH_LLAMA_TRACE=1 in the environment the
reference times each MUL_MAT_ID kernel with CUDA events and prints a SABAH_EV
line (per-call microseconds of gate/up and down calls) to stderr at exit.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
c_vp, c_sz, c_i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int


def load():
    L = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libsabah_rt_ref.so"))
    sig = {
        "sabah_rt_init": ([c_i], c_i),
        "sabah_rt_last_error": ([], ctypes.c_char_p),
        "sabah_rt_build_info": ([], ctypes.c_char_p),
        "sabah_rt_mul_mat_id_v2": ([c_vp, c_sz, c_sz, c_vp, c_sz, c_i, c_sz, c_vp, c_sz, c_sz, c_i, c_i,
                                    c_vp, c_sz, c_sz, c_i, c_i, c_i, c_i, c_vp, c_vp], c_i),
        "sabah_moe_block": ([c_vp, c_vp, c_vp, c_vp, c_vp, c_i, c_i, c_i, c_i, c_i, c_i, c_i], c_i),
        "sabah_dev_alloc": ([c_sz], c_vp),
        "sabah_memcpy_h2d": ([c_vp, c_vp, c_sz], c_i),
        "sabah_memcpy_d2h": ([c_vp, c_vp, c_sz], c_i),
        "sabah_sync_all": ([], c_i),
    }
    for name, (a, r) in sig.items():
        f = getattr(L, name)
        f.argtypes, f.restype = a, r
    return L


def check(L, rc, what):
    if rc != 0:
        raise RuntimeError("%s: %s" % (what, L.sabah_rt_last_error().decode()))


def upload(L, arr):
    arr = np.ascontiguousarray(arr)
    p = L.sabah_dev_alloc(arr.nbytes)
    assert p, "sabah_dev_alloc"
    check(L, L.sabah_memcpy_h2d(p, arr.ctypes.data, arr.nbytes), "h2d")
    return p


def main(mode: str, inp: str, outp: str, reps: int) -> None:
    L = load()
    check(L, L.sabah_rt_init(0), "sabah_rt_init")
    d = np.load(inp)
    if mode == "mmid":
        src = np.ascontiguousarray(d["source"])
        x = np.ascontiguousarray(d["x"], dtype=np.float32)
        ids = np.ascontiguousarray(d["ids"], dtype=np.int32)
        rows, k, E, qt = (int(d[n]) for n in ("rows", "k", "E", "qt"))
        T, x_rows, _ = x.shape
        n_ids = ids.shape[1]
        rb = src.shape[1] // rows
        d_x, d_ids = upload(L, x), upload(L, ids)
        out = np.zeros((T, n_ids, rows), np.float32)
        d_dst = L.sabah_dev_alloc(out.nbytes)
        for _ in range(reps + 1):
            check(L, L.sabah_rt_mul_mat_id_v2(src.ctypes.data, rows * rb, rb, d_x, k * 4, x_rows, x_rows * k * 4,
                                              d_ids, 4, n_ids * 4, n_ids, T, d_dst, rows * 4, n_ids * rows * 4,
                                              rows, k, E, qt, None, None), "sabah_rt_mul_mat_id_v2")
        check(L, L.sabah_sync_all(), "sync")
        check(L, L.sabah_memcpy_d2h(out.ctypes.data, d_dst, out.nbytes), "d2h")
    else:
        gate, up, down = (np.ascontiguousarray(d[n]) for n in ("gate", "up", "down"))
        ids = np.asarray(d["ids"], np.int64)
        w = np.ascontiguousarray(d["w"], dtype=np.float32)
        x = np.ascontiguousarray(d["x"], dtype=np.float32)
        d_model, ff = (int(d[n]) for n in ("d_model", "ff"))
        qg, qu, qd = (int(v) for v in d["qts"])
        n = len(ids)
        bg, bu, bd = upload(L, gate), upload(L, up), upload(L, down)
        gs, ds = gate.shape[1], down.shape[1]
        ptrs = np.array([bg + int(e) * gs for e in ids] + [bu + int(e) * gs for e in ids] +
                        [bd + int(e) * ds for e in ids], np.uint64)
        d_ptrs, d_w, d_x = upload(L, ptrs), upload(L, w), upload(L, x)
        out = np.zeros(d_model, np.float32)
        d_out = upload(L, out)
        d_h = L.sabah_dev_alloc(n * ff * 4)
        for _ in range(reps + 1):
            check(L, L.sabah_moe_block(d_x, d_out, d_h, d_ptrs, d_w, d_model, ff, n, qg, qu, qd, 0),
                  "sabah_moe_block")
        check(L, L.sabah_sync_all(), "sync")
        check(L, L.sabah_memcpy_d2h(out.ctypes.data, d_out, out.nbytes), "d2h")
    np.savez(outp, out=out, build_info=np.array(L.sabah_rt_build_info().decode()))


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2], sys.argv[3], int(sys.argv[4]))
