"""The fused routed block on the GPU: sabah_moe_block (reference ABI, pointer
table, one token) and sabah_moe_block_ids (device-resident banks, T tokens),
against the float64 reference_block (sabah/runtime/executor.py:134-159).
Reference test: sabah/tests/test_moe_block.py (agreement < 1e-5 rel-L2,
wrong-expert discrimination).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3
TIGHT = 2e-5


def _golden_block(golden, bname):
    p = "block_%s_" % bname
    return {k: golden[p + k] for k in ("gate", "up", "down", "ids", "w", "x", "want", "types")}


@pytest.mark.parametrize("bname", ["iq3s", "q4k_q6k"])
def test_reference_abi_block_matches_fp64(gpu_rt, orc, golden, bname):
    from sabah_moe_accelerator_b200 import rt
    b = _golden_block(golden, bname)
    qg, qu, qd = [int(v) for v in b["types"]]
    d_model, ff, n = 256, 256, len(b["ids"])
    banks = {r: torch.from_numpy(np.ascontiguousarray(b[r]).reshape(-1)).cuda() for r in ("gate", "up", "down")}
    strides = {r: b[r].shape[1] for r in ("gate", "up", "down")}
    ptrs = [banks[r].data_ptr() + int(e) * strides[r] for r in ("gate", "up", "down") for e in b["ids"]]
    d_ptrs = torch.tensor(ptrs, dtype=torch.int64, device="cuda")
    d_w = torch.from_numpy(b["w"]).cuda()
    d_x = torch.from_numpy(b["x"]).cuda()
    d_out = torch.full((d_model,), 7.0, device="cuda")
    d_h = torch.empty(n * ff, device="cuda")
    torch.cuda.synchronize()
    L = gpu_rt
    rt.check(L.sabah_moe_block(d_x.data_ptr(), d_out.data_ptr(), d_h.data_ptr(), d_ptrs.data_ptr(), d_w.data_ptr(),
                               d_model, ff, n, qg, qu, qd, 0), "moe_block")
    rt.check(L.sabah_sync_compute(), "sync")
    got = d_out.cpu().numpy()
    r = orc.rel_l2(got, b["want"])
    assert r <= TOL and r <= TIGHT, r
    # accumulate: out += y
    rt.check(L.sabah_moe_block(d_x.data_ptr(), d_out.data_ptr(), d_h.data_ptr(), d_ptrs.data_ptr(), d_w.data_ptr(),
                               d_model, ff, n, qg, qu, qd, 1), "moe_block acc")
    rt.check(L.sabah_sync_compute(), "sync")
    assert orc.rel_l2(d_out.cpu().numpy(), 2 * b["want"]) <= TIGHT
    # discrimination: one routed expert swapped for another must be far off
    wrong = [int(e) for e in b["ids"]]
    wrong[0] = next(e for e in range(b["gate"].shape[0]) if e not in wrong)
    ptrs = [banks[r].data_ptr() + e * strides[r] for r in ("gate", "up", "down") for e in wrong]
    d_ptrs.copy_(torch.tensor(ptrs, dtype=torch.int64))
    torch.cuda.synchronize()
    rt.check(L.sabah_moe_block(d_x.data_ptr(), d_out.data_ptr(), d_h.data_ptr(), d_ptrs.data_ptr(), d_w.data_ptr(),
                               d_model, ff, n, qg, qu, qd, 0), "moe_block wrong")
    rt.check(L.sabah_sync_compute(), "sync")
    assert orc.rel_l2(d_out.cpu().numpy(), b["want"]) > 100 * TIGHT


@pytest.mark.parametrize("qg,qd,T", [(21, 21, 1), (21, 21, 4), (12, 14, 4), (8, 8, 1)])
def test_block_ids_config_shape(gpu_rt, orc, qg, qd, T):
    """d_model 2048, ff 768, top-10 of 64 experts, T tokens, banks on the device."""
    from sabah_moe_accelerator_b200 import ops, rt
    d_model, ff, E, K = 2048, 768, 64, 10
    gate = ops.synth_rows(E * ff, d_model, qg, seed=31, sigma=0.02)
    up = ops.synth_rows(E * ff, d_model, qg, seed=32, sigma=0.02)
    down = ops.synth_rows(E * d_model, ff, qd, seed=33, sigma=0.02)
    rng = np.random.default_rng(T)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    x = rng.standard_normal((T, d_model)).astype(np.float32)
    out = ops.moe_block_ids(gate, up, down, torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(),
                            torch.from_numpy(x).cuda(), d_model, ff, E, qg, qg, qd)
    got = out.cpu().numpy()
    g, u, d = gate.cpu().numpy(), up.cpu().numpy(), down.cpu().numpy()
    for t in range(T):
        want = orc.moe_block_f64(g.reshape(E, -1), u.reshape(E, -1), d.reshape(E, -1), ids[t], w[t], x[t],
                                 d_model, ff, qg, qg, qd)
        r = orc.rel_l2(got[t], want)
        assert r <= TOL and r <= TIGHT, (t, r)


def test_block_ids_shape_changes(gpu_rt, orc):
    """Scratch reuse across shapes: T = 4, then a smaller T = 1, then T = 4 again,
    each against fp64 (the block's scratch is sized by the largest call so far)."""
    from sabah_moe_accelerator_b200 import ops
    d_model, ff, E, K, qt = 2048, 768, 32, 10, 21
    gate = ops.synth_rows(E * ff, d_model, qt, seed=41, sigma=0.02)
    up = ops.synth_rows(E * ff, d_model, qt, seed=42, sigma=0.02)
    down = ops.synth_rows(E * d_model, ff, qt, seed=43, sigma=0.02)
    g, u, d = gate.cpu().numpy(), up.cpu().numpy(), down.cpu().numpy()
    for case, T in enumerate((4, 1, 4)):
        rng = np.random.default_rng(300 + case)
        ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
        w = rng.random((T, K)).astype(np.float32)
        w /= w.sum(1, keepdims=True)
        x = rng.standard_normal((T, d_model)).astype(np.float32)
        out = ops.moe_block_ids(gate, up, down, torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(),
                                torch.from_numpy(x).cuda(), d_model, ff, E, qt, qt, qt)
        got = out.cpu().numpy()
        for t in range(T):
            want = orc.moe_block_f64(g.reshape(E, -1), u.reshape(E, -1), d.reshape(E, -1), ids[t], w[t], x[t],
                                     d_model, ff, qt, qt, qt)
            r = orc.rel_l2(got[t], want)
            assert r <= TOL and r <= TIGHT, (case, T, t, r)


@pytest.mark.parametrize("T", [40, 104])
def test_block_ids_grouped_path(gpu_rt, orc, T):
    """T x top-10 >= 384 (token, slot) pairs: the block runs as grouped gate / up
    / down MUL_MAT_IDs + SwiGLU + combine; against fp64 (sampled tokens), then
    with accumulate."""
    from sabah_moe_accelerator_b200 import ops
    d_model, ff, E, K, qt = 2048, 768, 24, 10, 21
    gate = ops.synth_rows(E * ff, d_model, qt, seed=61, sigma=0.02)
    up = ops.synth_rows(E * ff, d_model, qt, seed=62, sigma=0.02)
    down = ops.synth_rows(E * d_model, ff, qt, seed=63, sigma=0.02)
    rng = np.random.default_rng(400 + T)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    x = rng.standard_normal((T, d_model)).astype(np.float32)
    ids_d, w_d, x_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    out = ops.moe_block_ids(gate, up, down, ids_d, w_d, x_d, d_model, ff, E, qt, qt, qt)
    got = out.cpu().numpy()
    g, u, d = gate.cpu().numpy(), up.cpu().numpy(), down.cpu().numpy()
    sample = [0, 1, T // 2, T - 1]
    want = np.stack([orc.moe_block_f64(g.reshape(E, -1), u.reshape(E, -1), d.reshape(E, -1), ids[t], w[t], x[t],
                                       d_model, ff, qt, qt, qt) for t in sample])
    for j, t in enumerate(sample):
        r = orc.rel_l2(got[t], want[j])
        assert r <= TOL and r <= TIGHT, (t, r)
    ops.moe_block_ids(gate, up, down, ids_d, w_d, x_d, d_model, ff, E, qt, qt, qt, out=out, accumulate=True)
    torch.cuda.synchronize()
    assert orc.rel_l2(out.cpu().numpy(), 2 * got) <= TIGHT


@pytest.mark.parametrize("T,E", [(80, 64), (7, 16)])
def test_block_ids_one_slot_per_token(gpu_rt, orc, T, E):
    """n_used = 1 (the expert-parallel bank's per-pair call): the one-launch path
    takes 32 down rows of the single slot per item; against fp64, accumulate."""
    from sabah_moe_accelerator_b200 import ops
    d_model, ff, qt = 2048, 768, 21
    gate = ops.synth_rows(E * ff, d_model, qt, seed=71, sigma=0.02)
    up = ops.synth_rows(E * ff, d_model, qt, seed=72, sigma=0.02)
    down = ops.synth_rows(E * d_model, ff, qt, seed=73, sigma=0.02)
    rng = np.random.default_rng(T)
    ids = rng.integers(0, E, (T, 1)).astype(np.int32)
    w = (rng.random((T, 1)) + 0.5).astype(np.float32)
    x = rng.standard_normal((T, d_model)).astype(np.float32)
    ids_d, w_d, x_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    out = ops.moe_block_ids(gate, up, down, ids_d, w_d, x_d, d_model, ff, E, qt, qt, qt)
    got = out.cpu().numpy()
    g, u, d = (b.cpu().numpy().reshape(E, -1) for b in (gate, up, down))
    for t in sorted({0, T // 2, T - 1}):
        want = orc.moe_block_f64(g, u, d, ids[t], w[t], x[t], d_model, ff, qt, qt, qt)
        r = orc.rel_l2(got[t], want)
        assert r <= TOL and r <= TIGHT, (t, r)
    acc = x_d.clone()
    ops.moe_block_ids(gate, up, down, ids_d, w_d, x_d, d_model, ff, E, qt, qt, qt, out=acc, accumulate=True)
    torch.cuda.synchronize()
    assert orc.rel_l2(acc.cpu().numpy(), x + got) <= TIGHT


@pytest.mark.parametrize("qt,P,E", [(21, 80, 64), (21, 640, 64), (12, 40, 16)])
def test_block_gather_matches_block_on_gathered_rows(gpu_rt, orc, qt, P, E):
    """sabah_moe_block_gather (token t reads row xrows[t] of x) equals
    sabah_moe_block_ids on the gathered rows: in place on the one-launch IQ3_S
    path (80 pairs), through its gather pass elsewhere (grouped, Q4_K/Q6_K)."""
    import ctypes
    from sabah_moe_accelerator_b200 import ops, rt
    d_model, ff = 2048, 768
    qd = 14 if qt == 12 else qt
    n_used = 1 if qt == 21 else 10
    T = P if qt == 21 else P // n_used
    gate = ops.synth_rows(E * ff, d_model, qt, seed=81, sigma=0.02)
    up = ops.synth_rows(E * ff, d_model, qt, seed=82, sigma=0.02)
    down = ops.synth_rows(E * d_model, ff, qd, seed=83, sigma=0.02)
    rng = np.random.default_rng(P)
    n_rows = 37
    x_all = torch.from_numpy(rng.standard_normal((n_rows, d_model)).astype(np.float32)).cuda()
    rows = torch.from_numpy(rng.integers(0, n_rows, T).astype(np.int32)).cuda()
    ids = torch.from_numpy(np.stack([rng.choice(E, n_used, replace=False) for _ in range(T)]).astype(np.int32)).cuda()
    w = torch.from_numpy((rng.random((T, n_used)) + 0.5).astype(np.float32)).cuda()
    want = ops.moe_block_ids(gate, up, down, ids, w, x_all[rows.long()].contiguous(), d_model, ff, E, qt, qt, qd)
    out = torch.empty((T, d_model), device="cuda")
    h = torch.empty((T, n_used, ff), device="cuda")
    L = gpu_rt
    gs, ds = ff * rt.row_bytes(qt, d_model), d_model * rt.row_bytes(qd, ff)

    def call(rws):
        return L.sabah_moe_block_gather(ctypes.c_void_p(gate.data_ptr()), ctypes.c_void_p(up.data_ptr()),
                                        ctypes.c_void_p(down.data_ptr()), gs, ds, E, ctypes.c_void_p(ids.data_ptr()),
                                        ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(x_all.data_ptr()),
                                        ctypes.c_void_p(rws.data_ptr()), n_rows, ctypes.c_void_p(out.data_ptr()),
                                        ctypes.c_void_p(h.data_ptr()), d_model, ff, n_used, T, qt, qt, qd, 0,
                                        ctypes.c_void_p(ops._stream(None)))

    rt.check(call(rows), "sabah_moe_block_gather")
    torch.cuda.synchronize()
    assert orc.rel_l2(out.cpu().numpy(), want.cpu().numpy()) <= TIGHT
    assert L.sabah_rt_device_error() == 0
    bad = rows.clone()
    bad[1] = n_rows
    rt.check(call(bad), "sabah_moe_block_gather, bad row")
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    assert np.isnan(o[1]).all() and np.isfinite(o[0]).all()
    assert L.sabah_rt_device_error() == 1
