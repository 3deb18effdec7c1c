"""Expert-parallel bank on the GPU (sabah_moe_accelerator_b200/ep.py): the
sharded decode must match the single-GPU persistent decode (sabah_moe_decode)
and the fp64 chain of reference_block (sabah/runtime/executor.py:134-159).
world = 1 runs everywhere; the 2-rank case runs when two GPUs are visible."""
from __future__ import annotations

import ctypes
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3
TIGHT = 2e-5
QT = 21
D, F, E, K, T, LAYERS = 2048, 768, 32, 10, 8, 2
HERE = os.path.dirname(os.path.abspath(__file__))


def problem(e0=0, e1=E):
    """Experts [e0, e1) of the shared bank (the same bytes whatever the split),
    routing and x of the shared problem."""
    from sabah_moe_accelerator_b200 import ops, rt
    banks = []
    for L in range(LAYERS):
        parts = []
        for role, rows, k in ((0, F, D), (1, F, D), (2, D, F)):
            t = torch.empty((e1 - e0) * rows * rt.row_bytes(QT, k), dtype=torch.uint8, device="cuda")
            rt.check(rt.lib().sabah_synth_rows_at(ctypes.c_void_p(t.data_ptr()), QT, e0 * rows, (e1 - e0) * rows, k,
                                                  100 + 3 * L + role, 0.02, ctypes.c_void_p(ops._stream(None))),
                     "synth")
            parts.append(t)
        banks.append(tuple(parts))
    rng = np.random.default_rng(5)
    ids = np.stack([np.stack([rng.choice(E, K, replace=False) for _ in range(T)]) for _ in range(LAYERS)]).astype(np.int32)
    w = rng.random((LAYERS, T, K)).astype(np.float32)
    w /= w.sum(2, keepdims=True)
    x0 = rng.standard_normal((T, D)).astype(np.float32)
    torch.cuda.synchronize()
    return banks, ids, w, x0


def _single_gpu_reference(banks, ids, w, x0):
    from sabah_moe_accelerator_b200 import ops, rt
    arr = ctypes.c_void_p * LAYERS
    G, U, Dn = arr(*[b[0].data_ptr() for b in banks]), arr(*[b[1].data_ptr() for b in banks]), arr(*[b[2].data_ptr() for b in banks])
    x = torch.from_numpy(x0).cuda()
    h = torch.empty((T, K, F), device="cuda")
    ids_d, w_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    rt.check(rt.lib().sabah_moe_decode(LAYERS, G, U, Dn, F * rt.row_bytes(QT, D), D * rt.row_bytes(QT, F), E,
                                       ctypes.c_void_p(ids_d.data_ptr()), ctypes.c_void_p(w_d.data_ptr()),
                                       ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(h.data_ptr()), D, F, K, T,
                                       QT, QT, QT, ctypes.c_void_p(ops._stream(None))), "sabah_moe_decode")
    torch.cuda.synchronize()
    return x.cpu().numpy()


@pytest.mark.parametrize("exchange", ["ag", "a2a"])
def test_ep_world1_matches_decode_and_fp64(gpu_rt, orc, exchange):
    from sabah_moe_accelerator_b200 import ep
    banks, ids, w, x0 = problem()
    if exchange == "ag":
        plans = ep.pack_plans([ep.plan_layer(ids[L], w[L], 0, 1, E) for L in range(LAYERS)])
    else:
        plans = ep.pack_plans_a2a([ep.plan_layer_a2a(ids[L], w[L], 0, 1, E) for L in range(LAYERS)])
    x = torch.from_numpy(x0).cuda()
    ep.decode_step(x, plans, ep.CudaOps(banks, D, F, E, QT), ep.SingleComm(), exchange)
    torch.cuda.synchronize()
    got = x.cpu().numpy()
    assert gpu_rt.sabah_rt_device_error() == 0
    ref = _single_gpu_reference(banks, ids, w, x0)
    host = [tuple(t.cpu().numpy().reshape(E, -1) for t in b) for b in banks]
    want = x0.astype(np.float64)
    for L in range(LAYERS):
        g, u, d = host[L]
        want = np.stack([want[t] + orc.moe_block_f64(g, u, d, ids[L, t], w[L, t], want[t].astype(np.float32), D, F,
                                                     QT, QT, QT) for t in range(T)])
    for t in range(T):
        r = orc.rel_l2(got[t], want[t])
        assert r <= TOL and r <= TIGHT, ("fp64", t, r)
        assert orc.rel_l2(got[t], ref[t]) <= TIGHT, ("decode", t)


def test_ep_sum_rows_and_gather_edges(gpu_rt):
    """Empty pair lists give zero rows; out-of-range gather rows give zero rows."""
    from sabah_moe_accelerator_b200 import ep
    ops_ = ep.CudaOps([], D, F, E, QT)
    y = torch.full((3, D), 5.0, device="cuda")
    ops_.sum_rows(None, torch.zeros(4, dtype=torch.int32, device="cuda"), y)
    src = torch.randn(2, D, device="cuda")
    dst = torch.full((3, D), 5.0, device="cuda")
    ops_.gather(src, torch.tensor([1, 7, -1], dtype=torch.int32, device="cuda"), dst)
    torch.cuda.synchronize()
    assert float(y.abs().sum()) == 0.0
    assert torch.equal(dst[0], src[1]) and float(dst[1:].abs().sum()) == 0.0


def test_ep_sum_rows_ex_residual_and_index(gpu_rt):
    """The fused pair sum: residual rows folded in (in place, or at a row
    offset), indexed sources, out-of-range indices add nothing."""
    from sabah_moe_accelerator_b200 import ep
    ops_ = ep.CudaOps([], D, F, E, QT)
    src = torch.randn(5, D, device="cuda")
    x = torch.randn(3, D, device="cuda")
    idx = torch.tensor([4, 0, 9, 2, -1], dtype=torch.int32, device="cuda")
    off = torch.tensor([0, 2, 2, 5], dtype=torch.int32, device="cuda")
    dst = x.clone()
    ops_.sum_rows_ex(src, 5, idx, off, dst, dst, 0)
    x1 = torch.randn(1, D, device="cuda")
    dst2 = torch.full((3, D), 9.0, device="cuda")
    ops_.sum_rows_ex(src, 5, None, torch.tensor([0, 1, 3, 5], dtype=torch.int32, device="cuda"), dst2, x1, 1)
    torch.cuda.synchronize()
    assert torch.allclose(dst[0], x[0] + src[4] + src[0]) and torch.equal(dst[1], x[1])
    assert torch.allclose(dst[2], x[2] + src[2])
    assert torch.allclose(dst2[0], src[0]) and torch.allclose(dst2[1], x1[0] + src[1] + src[2])
    assert torch.allclose(dst2[2], src[3] + src[4])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["ag", "a2a"])
def test_ep_two_ranks_match_single_gpu(gpu_rt, tmp_path, exchange):
    out = str(tmp_path / "ep")
    env = dict(os.environ, PYTHONPATH=HERE + os.pathsep + os.path.dirname(HERE))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=%d" % _free_port(), os.path.join(HERE, "ep_child.py"), out,
           exchange]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    got = np.concatenate([np.load("%s_%d.npy" % (out, k)) for k in range(2)])
    banks, ids, w, x0 = problem()
    ref = _single_gpu_reference(banks, ids, w, x0)
    for t in range(T):
        rel = float(np.linalg.norm(got[t] - ref[t]) / np.linalg.norm(ref[t]))
        assert rel <= TIGHT, (t, rel)
