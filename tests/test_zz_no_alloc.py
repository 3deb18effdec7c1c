"""sabah_moe_block_ids_noalloc (fixed device scratch, nothing allocated) against
sabah_moe_block_ids on the same inputs, both through the C ABI, and both
against the float64 oracle of the routed block (reference_block,
sabah/runtime/executor.py:134-159) over the same dequantized weights.

The file sorts last, so the in-process test runs after every other test has
used the runtime; the child test runs the same check in a fresh process, where
the first call does the per-device set-up.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3     # rel-L2 gate of the routed path against fp64
TIGHT = 2e-5   # same kernels on both sides: only summation order may differ
ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))


def _rel(a, b):
    return float(np.linalg.norm(a - b) / max(float(np.linalg.norm(b)), 1e-30))


def check(init: bool) -> None:
    import torch

    from oracle import cpu as orc
    from sabah_moe_accelerator_b200 import ops, rt
    if init:
        ops.init(0)
    L = rt.lib()
    d_model, ff, E, K = 2048, 768, 64, 10
    qt = rt.QTYPE["IQ3_S"]
    gate = ops.synth_rows(E * ff, d_model, qt, seed=51, sigma=0.02)
    up = ops.synth_rows(E * ff, d_model, qt, seed=52, sigma=0.02)
    down = ops.synth_rows(E * d_model, ff, qt, seed=53, sigma=0.02)
    gs, ds = ff * rt.row_bytes(qt, d_model), d_model * rt.row_bytes(qt, ff)
    gh, uh, dh = (t.cpu().numpy().reshape(E, -1) for t in (gate, up, down))
    st = ctypes.c_void_p(ops._stream(None))
    vp = ctypes.c_void_p

    def run(fn, T, ids, w, x, out, h, acc):
        return fn(vp(gate.data_ptr()), vp(up.data_ptr()), vp(down.data_ptr()), gs, ds, E, vp(ids.data_ptr()),
                  vp(w.data_ptr()), vp(x.data_ptr()), vp(out.data_ptr()), vp(h.data_ptr()), d_model, ff, K, T,
                  qt, qt, qt, acc, st)

    # T = 4 then 1 then 4 again: the counters' layout moves between shapes
    for case, T in enumerate((4, 1, 4)):
        rng = np.random.default_rng(200 + case)
        ids = torch.from_numpy(np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)).cuda()
        w = rng.random((T, K)).astype(np.float32)
        w = torch.from_numpy(w / w.sum(1, keepdims=True)).cuda()
        x = torch.from_numpy(rng.standard_normal((T, d_model)).astype(np.float32)).cuda()
        out_ref = torch.empty((T, d_model), device="cuda")
        h_ref = torch.empty((T, K, ff), device="cuda")
        rt.check(run(L.sabah_moe_block_ids, T, ids, w, x, out_ref, h_ref, 0), "sabah_moe_block_ids")
        torch.cuda.synchronize()
        want = out_ref.cpu().numpy()
        assert np.isfinite(want).all()
        ids_h, w_h, x_h = ids.cpu().numpy(), w.cpu().numpy(), x.cpu().numpy()
        exact = [orc.moe_block_f64(gh, uh, dh, ids_h[t], w_h[t], x_h[t], d_model, ff, qt, qt, qt) for t in range(T)]
        for call in range(2):   # two calls in a row
            out = torch.full((T, d_model), 7.0, device="cuda")
            h = torch.empty((T, K, ff), device="cuda")
            rt.check(run(L.sabah_moe_block_ids_noalloc, T, ids, w, x, out, h, 0), "sabah_moe_block_ids_noalloc")
            torch.cuda.synchronize()
            got = out.cpu().numpy()
            for t in range(T):
                r = _rel(got[t], want[t])
                assert r <= TOL and r <= TIGHT, (T, call, t, r)
                r64 = _rel(got[t].astype(np.float64), exact[t])
                assert r64 <= TOL, ("vs fp64", T, call, t, r64)
        # accumulate: out += y
        rt.check(run(L.sabah_moe_block_ids_noalloc, T, ids, w, x, out, h, 1), "noalloc accumulate")
        torch.cuda.synchronize()
        assert _rel(out.cpu().numpy(), 2 * want) <= TIGHT

    # beyond the fixed scratch: refused before any launch, with the limit named
    T = 8
    ids = torch.zeros((T, K), dtype=torch.int32, device="cuda")
    w = torch.zeros((T, K), device="cuda")
    x = torch.zeros((T, d_model), device="cuda")
    out = torch.zeros((T, d_model), device="cuda")
    h = torch.empty((T, K, ff), device="cuda")
    assert run(L.sabah_moe_block_ids_noalloc, T, ids, w, x, out, h, 0) == -1
    assert "fixed scratch" in rt.last_error()
    # the refusal came from the host: no kernel ran, no device error is pending
    torch.cuda.synchronize()
    assert L.sabah_rt_device_error() == 0


def test_noalloc_matches_block_ids(gpu_rt):
    check(init=False)


def test_noalloc_fresh_process():
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    r = subprocess.run([sys.executable, os.path.abspath(__file__)], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "noalloc ok" in r.stdout


if __name__ == "__main__":
    check(init=True)
    print("noalloc ok")
