"""Generate the committed golden fixtures (tests/golden/golden.npz).

Run in the build container, where gguf-py and the reference build
(oracle/_ref/libsabah_rt_ref.so, made by oracle/build_ref.sh) are available:

    python tests/golden/make_golden.py

Contents (all seeded, so the script reproduces the file):
  raw_<T>, gguf_<T>, ref_<T>  per quant type T: 16 random blocks (random bytes,
      scale fields set to finite fp16 values), their dequantization by gguf-py
      (gguf.quants.dequantize, the reference harness's dequant oracle) and by
      the reference's own sabah_rt_host_dequant. A type one side lacks is
      omitted for that side (Q6_K is not in the reference, Q2_0 not in gguf-py).
  mmid_<T>_<mode>_*  small MUL_MAT_ID cases: an expert tensor, ids, x and the
      float64 result W.x computed from gguf-py-dequantized weights with numpy.
  block_<name>_*  one fused MoE block (reference_block semantics) in float64.
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))

TYPES = {"Q5_1": 7, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ3_XXS": 18, "IQ4_NL": 20,
         "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "Q2_0": 42}
QBLOCK = {7: (32, 24), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210), 18: (256, 98),
          20: (32, 18), 21: (256, 110), 22: (256, 82), 23: (256, 136), 42: (64, 18)}
# byte offsets of the fp16 scale fields of each block layout
F16_FIELDS = {"Q5_1": [0, 2], "Q4_K": [0, 2], "Q5_K": [0, 2], "Q6_K": [208]}


def random_blocks(rng, name: str, n_blocks: int, scale: float = 0.01) -> np.ndarray:
    qt = TYPES[name]
    bb = QBLOCK[qt][1]
    raw = rng.integers(0, 256, size=(n_blocks, bb), dtype=np.uint8)
    for off in F16_FIELDS.get(name, [0]):
        d = (rng.standard_normal(n_blocks) * scale).astype(np.float16)
        raw[:, off:off + 2] = d.view(np.uint8).reshape(n_blocks, 2)
    return raw


def gguf_dequant(raw: np.ndarray, name: str) -> np.ndarray | None:
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as Q
    if not hasattr(Q, name):
        return None
    return np.asarray(quants.dequantize(raw, getattr(Q, name)), np.float32).reshape(-1)


def ref_dequant(raw: np.ndarray, name: str):
    path = os.path.join(ROOT, "oracle", "_ref", "libsabah_rt_ref.so")
    L = ctypes.CDLL(path)
    L.sabah_rt_host_dequant.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    qt = TYPES[name]
    n = raw.shape[0] * QBLOCK[qt][0]
    out = np.empty(n, np.float32)
    raw = np.ascontiguousarray(raw)
    return out if L.sabah_rt_host_dequant(raw.ctypes.data, out.ctypes.data, qt, n) == 0 else None


def dense_weights(raw_expert: np.ndarray, name: str, rows: int, k: int) -> np.ndarray:
    return gguf_dequant(raw_expert.reshape(-1, QBLOCK[TYPES[name]][1]), name).astype(np.float64).reshape(rows, k)


def main() -> None:
    rng = np.random.default_rng(20261201)
    out: dict[str, np.ndarray] = {}
    for name in TYPES:
        raw = random_blocks(rng, name, 16)
        out["raw_" + name] = raw
        g = gguf_dequant(raw, name)
        if g is not None:
            out["gguf_" + name] = g
        r = ref_dequant(raw, name)
        if r is not None:
            out["ref_" + name] = r

    # small MUL_MAT_ID cases (gguf-py dequant + numpy float64)
    E, rows, k, T, K = 6, 8, 512, 3, 4
    for name in ("IQ3_S", "Q8_0", "Q4_K", "Q6_K"):
        qt = TYPES[name]
        be, bb = QBLOCK[qt]
        rb = k // be * bb
        src = random_blocks(rng, name, E * rows * (k // be)).reshape(E, rows * rb)
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
        for mode, x_rows in (("bcast", 1), ("perslot", K)):
            x = rng.standard_normal((T, x_rows, k)).astype(np.float32)
            want = np.empty((T, K, rows), np.float64)
            for t in range(T):
                for i in range(K):
                    W = dense_weights(src[ids[t, i]], name, rows, k)
                    want[t, i] = W @ x[t, i % x_rows].astype(np.float64)
            p = "mmid_%s_%s_" % (name, mode)
            out[p + "src"], out[p + "ids"], out[p + "x"], out[p + "want"] = src, ids, x, want

    # fused blocks (reference_block in float64)
    d_model, ff, E, n_used = 256, 256, 4, 3
    for bname, (qg, qd) in {"iq3s": ("IQ3_S", "IQ3_S"), "q4k_q6k": ("Q4_K", "Q6_K")}.items():
        def bank(name, rws, kk):
            be, bb = QBLOCK[TYPES[name]]
            return random_blocks(rng, name, E * rws * (kk // be), 0.002).reshape(E, -1)
        gate, up, down = bank(qg, ff, d_model), bank(qg, ff, d_model), bank(qd, d_model, ff)
        ids = rng.choice(E, n_used, replace=False).astype(np.int32)
        w = rng.random(n_used).astype(np.float32)
        w /= w.sum()
        x = rng.standard_normal(d_model).astype(np.float32)
        y = np.zeros(d_model, np.float64)
        for wk, e in zip(w, ids):
            g = dense_weights(gate[e], qg, ff, d_model) @ x.astype(np.float64)
            u = dense_weights(up[e], qg, ff, d_model) @ x.astype(np.float64)
            h = g / (1.0 + np.exp(-g)) * u
            y += float(wk) * (dense_weights(down[e], qd, d_model, ff) @ h)
        p = "block_%s_" % bname
        out[p + "gate"], out[p + "up"], out[p + "down"] = gate, up, down
        out[p + "ids"], out[p + "w"], out[p + "x"], out[p + "want"] = ids, w, x, y
        out[p + "types"] = np.array([TYPES[qg], TYPES[qg], TYPES[qd]], np.int32)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print("wrote", os.path.join(HERE, "golden.npz"), sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    sys.exit(main())
