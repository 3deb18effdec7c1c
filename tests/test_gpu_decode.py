"""sabah_moe_decode: n_layers routed blocks with x <- x + block_L(x), one call
per decode step. IQ3_S shapes that fit run as one persistent launch; the
result must match the fp64 chain of reference_block
(sabah/runtime/executor.py:134-159, run_model :101-112) and the per-block
entry point (sabah_moe_block_ids, accumulate = 1) layer by layer.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3
TIGHT = 2e-5
QT = 21   # IQ3_S


def _banks(n_layers, E, d_model, ff, seed):
    from sabah_moe_accelerator_b200 import ops
    out = []
    for L in range(n_layers):
        g = ops.synth_rows(E * ff, d_model, QT, seed=seed + 3 * L, sigma=0.02)
        u = ops.synth_rows(E * ff, d_model, QT, seed=seed + 3 * L + 1, sigma=0.02)
        d = ops.synth_rows(E * d_model, ff, QT, seed=seed + 3 * L + 2, sigma=0.02)
        out.append((g, u, d))
    return out


def _decode(L, banks, ids, w, x, h, d_model, ff, E):
    from sabah_moe_accelerator_b200 import ops, rt
    n_layers = len(banks)
    T, K = ids.shape[1], ids.shape[2]
    arr = ctypes.c_void_p * n_layers
    G = arr(*[b[0].data_ptr() for b in banks])
    U = arr(*[b[1].data_ptr() for b in banks])
    D = arr(*[b[2].data_ptr() for b in banks])
    gs, ds = ff * rt.row_bytes(QT, d_model), d_model * rt.row_bytes(QT, ff)
    return L.sabah_moe_decode(n_layers, G, U, D, gs, ds, E, ctypes.c_void_p(ids.data_ptr()),
                              ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(x.data_ptr()),
                              ctypes.c_void_p(h.data_ptr()), d_model, ff, K, T, QT, QT, QT,
                              ctypes.c_void_p(ops._stream(None)))


@pytest.mark.parametrize("T,n_layers", [(1, 3), (2, 2), (4, 2)])
def test_decode_matches_fp64_chain_and_block_loop(gpu_rt, orc, T, n_layers):
    from sabah_moe_accelerator_b200 import ops, rt
    d_model, ff, E, K = 2048, 768, 32, 10
    banks = _banks(n_layers, E, d_model, ff, seed=500 + 10 * T)
    rng = np.random.default_rng(700 + T)
    ids = np.stack([[rng.choice(E, K, replace=False) for _ in range(T)] for _ in range(n_layers)]).astype(np.int32)
    w = rng.random((n_layers, T, K)).astype(np.float32)
    w /= w.sum(2, keepdims=True)
    x0 = rng.standard_normal((T, d_model)).astype(np.float32)
    ids_d, w_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    x = torch.from_numpy(x0).cuda()
    h = torch.empty((T, K, ff), device="cuda")
    L = gpu_rt
    rt.check(_decode(L, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode")
    torch.cuda.synchronize()
    got = x.cpu().numpy()
    assert L.sabah_rt_device_error() == 0

    # the per-block entry point, layer by layer, accumulating into x
    xb = torch.from_numpy(x0).cuda()
    for Lr in range(n_layers):
        ops.moe_block_ids(banks[Lr][0], banks[Lr][1], banks[Lr][2], ids_d[Lr].contiguous(), w_d[Lr].contiguous(),
                          xb.clone(), d_model, ff, E, QT, QT, QT, out=xb, accumulate=True)
    torch.cuda.synchronize()
    loop = xb.cpu().numpy()

    # fp64 chain
    host = [tuple(t.cpu().numpy().reshape(E, -1) for t in b) for b in banks]
    want = x0.astype(np.float64)
    for Lr in range(n_layers):
        g, u, d = host[Lr]
        want = np.stack([want[t] + orc.moe_block_f64(g, u, d, ids[Lr, t], w[Lr, t], want[t].astype(np.float32),
                                                     d_model, ff, QT, QT, QT) for t in range(T)])
    for t in range(T):
        r = orc.rel_l2(got[t], want[t])
        assert r <= TOL and r <= TIGHT, ("fp64", t, r)
        rb = orc.rel_l2(got[t], loop[t])
        assert rb <= TIGHT, ("block loop", t, rb)


def test_decode_out_of_range_id_is_reported(gpu_rt):
    from sabah_moe_accelerator_b200 import rt
    d_model, ff, E, K, T, n_layers = 2048, 768, 16, 10, 1, 2
    banks = _banks(n_layers, E, d_model, ff, seed=900)
    ids = np.tile(np.arange(K, dtype=np.int32), (n_layers, T, 1))
    ids[1, 0, 3] = E   # layer 1, slot 3: outside [0, E)
    ids_d = torch.from_numpy(ids).cuda()
    w_d = torch.full((n_layers, T, K), 0.1, device="cuda")
    x = torch.randn((T, d_model), device="cuda")
    h = torch.empty((T, K, ff), device="cuda")
    L = gpu_rt
    rt.check(_decode(L, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode")
    torch.cuda.synchronize()
    assert L.sabah_rt_device_error() == 1
    assert np.isnan(x.cpu().numpy()).any()
    # the error was read and cleared: the next call runs clean
    ids_d[1, 0, 3] = 0
    x.normal_()
    rt.check(_decode(L, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode after error")
    torch.cuda.synchronize()
    assert L.sabah_rt_device_error() == 0
    assert np.isfinite(x.cpu().numpy()).all()
