"""Q8_0 on the tensor-core matvec engine (csrc/sb_mmid_iq3s.cu, k_iq3s<8>):
int8 quants become exact fp16 (bias trick), x comes as the IQ3_S path's hi/lo
fp16 sets, 16-row tiles arrive as 8 row-pair bulk copies at a padded stride.
Every case must match the fp64 oracle at reference grade, and must have run on
the Q8_0 kernels (kernel timing names), not on the generic warp-per-row path.
Reference decoder: sub32_q8_0 (sabah/runtime/cuda/sabah_rt.cu:2537-2545); the
fused block's k_gate_up / k_down (:2725-2785).
"""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3
TIGHT = 2e-5
QT = 8


def _timed(fn):
    """Run fn with the library's kernel timing on; the names of what ran."""
    import ctypes
    from sabah_moe_accelerator_b200 import rt
    L = rt.lib()
    torch.cuda.synchronize()
    L.sabah_rt_kernel_timing(1)
    try:
        out = fn()
        torch.cuda.synchronize()
        buf = ctypes.create_string_buffer(8192)
        L.sabah_rt_kernel_times(buf, 8192)
    finally:
        L.sabah_rt_kernel_timing(0)
    return out, set(json.loads(buf.value.decode()))


@pytest.mark.parametrize("rows,k,T,x_rows", [
    (768, 2048, 1, 1),      # cfg 1 gate/up call
    (2048, 768, 1, 10),     # cfg 1 down call: one input row per slot
    (768, 2048, 3, 1),      # a few tokens
    (2048, 768, 2, 10),
    (128, 1024, 4, 1),      # another k (8 groups) and a 128-row matrix
])
def test_mmid_q8_0_matches_fp64(gpu_rt, orc, rows, k, T, x_rows):
    from sabah_moe_accelerator_b200 import ops, rt
    E, K = 48, 10
    rb = rt.row_bytes(QT, k)
    bank = ops.synth_rows(E * rows, k, QT, seed=rows + k, sigma=0.02)
    rng = np.random.default_rng(rows * 3 + T)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    x = rng.standard_normal((T, x_rows, k)).astype(np.float32)
    d_x, d_ids = torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda()
    out, names = _timed(lambda: ops.mul_mat_id(bank, rows * rb, rb, d_x, d_ids, rows, k, E, QT))
    assert "mmid_q8_0" in names, names
    want = orc.mmid_f64(bank.cpu().numpy(), rows * rb, rb, x, x_rows, ids, rows, k, E, QT)
    got = out.cpu().numpy().astype(np.float64)
    for t in range(T):
        for i in range(K):
            r = np.linalg.norm(got[t, i] - want[t, i]) / np.linalg.norm(want[t, i])
            assert r <= TOL and r <= TIGHT, (t, i, r)


@pytest.mark.parametrize("T", [1, 3])
def test_block_q8_0_matches_fp64(gpu_rt, orc, T):
    """The cfg 1 block shape (d_model 2048, ff 768, top-10) on device banks."""
    from sabah_moe_accelerator_b200 import ops
    d_model, ff, E, K = 2048, 768, 96, 10
    gate = ops.synth_rows(E * ff, d_model, QT, seed=41, sigma=0.02)
    up = ops.synth_rows(E * ff, d_model, QT, seed=42, sigma=0.02)
    down = ops.synth_rows(E * d_model, ff, QT, seed=43, sigma=0.02)
    rng = np.random.default_rng(40 + T)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    w /= w.sum(1, keepdims=True)
    x = rng.standard_normal((T, d_model)).astype(np.float32)
    out, names = _timed(lambda: ops.moe_block_ids(gate, up, down, torch.from_numpy(ids).cuda(),
                                                  torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda(),
                                                  d_model, ff, E, QT, QT, QT))
    assert {"gate_up_q8_0", "down_q8_0"} <= names, names
    got = out.cpu().numpy()
    g, u, d = gate.cpu().numpy(), up.cpu().numpy(), down.cpu().numpy()
    for t in range(T):
        want = orc.moe_block_f64(g.reshape(E, -1), u.reshape(E, -1), d.reshape(E, -1), ids[t], w[t], x[t],
                                 d_model, ff, QT, QT, QT)
        r = orc.rel_l2(got[t], want)
        assert r <= TOL and r <= TIGHT, (t, r)


def test_mmid_q8_0_out_of_range_id(gpu_rt):
    """A bad id on the fast path: that slot is NaN, the others exact, and the
    device error word reports it on the next call."""
    from sabah_moe_accelerator_b200 import ops, rt
    rows, k, E = 768, 2048, 8
    rb = rt.row_bytes(QT, k)
    bank = ops.synth_rows(E * rows, k, QT, seed=7)
    ids = torch.tensor([[0, E, 3]], dtype=torch.int32, device="cuda")
    x = torch.randn(1, 1, k, device="cuda")
    out, names = _timed(lambda: ops.mul_mat_id(bank, rows * rb, rb, x, ids, rows, k, E, QT))
    assert "mmid_q8_0" in names, names
    o = out.cpu().numpy()
    assert np.isfinite(o[0, 0]).all() and np.isnan(o[0, 1]).all() and np.isfinite(o[0, 2]).all()
    with pytest.raises(rt.SabahCudaError, match="outside"):
        ops.mul_mat_id(bank, rows * rb, rb, x, ids[:, :1].contiguous(), rows, k, E, QT)
    assert rt.lib().sabah_rt_device_error() == 0
