"""The barrier-free one-token IQ3_S decode (sb_flow_iq3s.cu), reached through
sabah_moe_decode and sabah_moe_block_ids with one token. Every case is checked
against the fp64 chain of reference_block (sabah/runtime/executor.py:134-159,
run_model :101-112) over the same dequantized weights, including the
benchmark's own bank (48 blocks x 512 experts) and routing set 0.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

TOL = 2e-3    # rel-L2 gate against fp64 (north_star tolerance)
TIGHT = 2e-5  # what the kernel delivers in practice (~1e-7 .. 1e-6)
QT = 21       # IQ3_S


def _banks(n_layers, E, d_model, ff, seed):
    from sabah_moe_accelerator_b200 import ops
    return [tuple(ops.synth_rows(E * rows, k, QT, seed=seed + 3 * L + role, sigma=0.02)
                  for role, (rows, k) in enumerate(((ff, d_model), (ff, d_model), (d_model, ff))))
            for L in range(n_layers)]


def _decode(L, banks, ids, w, x, h, d_model, ff, E):
    from sabah_moe_accelerator_b200 import ops, rt
    n = len(banks)
    arr = ctypes.c_void_p * n
    G, U, D = (arr(*[b[r].data_ptr() for b in banks]) for r in range(3))
    gs, ds = ff * rt.row_bytes(QT, d_model), d_model * rt.row_bytes(QT, ff)
    return L.sabah_moe_decode(n, G, U, D, gs, ds, E, ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                              ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(h.data_ptr()), d_model, ff,
                              ids.shape[-1], 1, QT, QT, QT, ctypes.c_void_p(ops._stream(None)))


def _routed(bank, ids, per_expert):
    """The routed experts' bytes (in slot order) as a compact host bank."""
    return np.stack([bank[int(i) * per_expert:(int(i) + 1) * per_expert].cpu().numpy() for i in ids])


def _chain_f64(orc, banks, ids, w, x0, d_model, ff):
    from sabah_moe_accelerator_b200 import rt
    gs, ds = ff * rt.row_bytes(QT, d_model), d_model * rt.row_bytes(QT, ff)
    want = x0.astype(np.float64)
    K = ids.shape[-1]
    for L, (g, u, d) in enumerate(banks):
        gh, uh, dh = _routed(g, ids[L], gs), _routed(u, ids[L], gs), _routed(d, ids[L], ds)
        want = want + orc.moe_block_f64(gh, uh, dh, np.arange(K, dtype=np.int32), w[L], want.astype(np.float32),
                                        d_model, ff, QT, QT, QT)
    return want


def _routing(rng, n_layers, E, K):
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(n_layers)]).astype(np.int32)
    w = rng.random((n_layers, K)).astype(np.float32)
    return ids, w / w.sum(1, keepdims=True)


@pytest.mark.parametrize("E,K,n_layers", [(512, 10, 6), (64, 1, 3), (64, 3, 2), (48, 16, 2)])
def test_flow_decode_matches_fp64_chain(gpu_rt, orc, E, K, n_layers):
    d_model, ff = 2048, 768
    banks = _banks(n_layers, E, d_model, ff, seed=3000 + E + K)
    rng = np.random.default_rng(E * 7 + K)
    ids, w = _routing(rng, n_layers, E, K)
    x0 = rng.standard_normal(d_model).astype(np.float32)
    x = torch.from_numpy(x0).cuda().view(1, -1)
    h = torch.empty((1, K, ff), device="cuda")
    ids_d, w_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    from sabah_moe_accelerator_b200 import rt
    rt.check(_decode(gpu_rt, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode")
    torch.cuda.synchronize()
    assert gpu_rt.sabah_rt_device_error() == 0
    got = x.cpu().numpy()[0]
    want = _chain_f64(orc, banks, ids, w, x0, d_model, ff)
    r = orc.rel_l2(got, want)
    assert r <= TOL and r <= TIGHT, r
    # h is the last block's: silu(gate . x) * (up . x) of each slot
    assert np.isfinite(h.cpu().numpy()).all()


def test_flow_repeated_launches_are_identical(gpu_rt):
    """Launch after launch on the same inputs gives the same bits: the tags of
    one launch are never taken for another's (the epoch advances per launch)."""
    d_model, ff, E, K, n_layers = 2048, 768, 64, 10, 4
    banks = _banks(n_layers, E, d_model, ff, seed=4100)
    rng = np.random.default_rng(41)
    ids, w = _routing(rng, n_layers, E, K)
    ids_d, w_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    x0 = torch.randn((1, d_model), device="cuda")
    h = torch.empty((1, K, ff), device="cuda")
    outs = []
    from sabah_moe_accelerator_b200 import rt
    for _ in range(4):
        x = x0.clone()
        rt.check(_decode(gpu_rt, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode")
        outs.append(x)
    # and a different routing in between must not leak into the next launch
    x_other = x0.clone()
    rt.check(_decode(gpu_rt, banks, torch.flip(ids_d, [1]).contiguous(), w_d, x_other, h, d_model, ff, E), "decode")
    x = x0.clone()
    rt.check(_decode(gpu_rt, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode")
    outs.append(x)
    torch.cuda.synchronize()
    ref = outs[0].cpu().numpy()
    for o in outs[1:]:
        assert np.array_equal(o.cpu().numpy(), ref)
    assert not np.array_equal(x_other.cpu().numpy(), ref)


def test_flow_bad_id_gives_nan_and_error_then_recovers(gpu_rt):
    d_model, ff, E, K, n_layers = 2048, 768, 32, 10, 3
    banks = _banks(n_layers, E, d_model, ff, seed=4200)
    ids = np.tile(np.arange(K, dtype=np.int32), (n_layers, 1))
    ids[1, 4] = E + 3
    ids_d = torch.from_numpy(ids).cuda()
    w_d = torch.full((n_layers, K), 0.1, device="cuda")
    x = torch.randn((1, d_model), device="cuda")
    h = torch.empty((1, K, ff), device="cuda")
    from sabah_moe_accelerator_b200 import rt
    rt.check(_decode(gpu_rt, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode")
    torch.cuda.synchronize()
    assert gpu_rt.sabah_rt_device_error() == 1
    assert np.isnan(x.cpu().numpy()).all()   # layer 1's y is NaN in every row, so is every later x
    ids_d[1, 4] = 0
    x.normal_()
    rt.check(_decode(gpu_rt, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode")
    torch.cuda.synchronize()
    assert gpu_rt.sabah_rt_device_error() == 0
    assert np.isfinite(x.cpu().numpy()).all()


@pytest.mark.parametrize("accumulate", [False, True])
def test_flow_single_block(gpu_rt, orc, accumulate):
    """sabah_moe_block_ids with one token runs the same kernel as one block:
    out = (accumulate ? out : 0) + y, x untouched."""
    from sabah_moe_accelerator_b200 import ops
    d_model, ff, E, K = 2048, 768, 128, 10
    (g, u, d), = _banks(1, E, d_model, ff, seed=4300)
    rng = np.random.default_rng(43)
    ids, w = _routing(rng, 1, E, K)
    x = torch.from_numpy(rng.standard_normal((1, d_model)).astype(np.float32)).cuda()
    out0 = torch.from_numpy(rng.standard_normal((1, d_model)).astype(np.float32)).cuda()
    out = out0.clone()
    x_before = x.clone()
    ops.moe_block_ids(g, u, d, torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), x, d_model, ff, E, QT, QT,
                      QT, out=out, accumulate=accumulate)
    torch.cuda.synchronize()
    assert torch.equal(x, x_before)
    from sabah_moe_accelerator_b200 import rt
    gs, ds = ff * rt.row_bytes(QT, d_model), d_model * rt.row_bytes(QT, ff)
    y = orc.moe_block_f64(_routed(g, ids[0], gs), _routed(u, ids[0], gs), _routed(d, ids[0], ds),
                          np.arange(K, dtype=np.int32), w[0], x.cpu().numpy()[0], d_model, ff, QT, QT, QT)
    want = y + (out0.cpu().numpy()[0].astype(np.float64) if accumulate else 0.0)
    r = orc.rel_l2(out.cpu().numpy()[0], want)
    assert r <= TOL and r <= TIGHT, r


def test_flow_matches_phase_barrier_kernel():
    """The same decode with the barrier-free kernel switched off
    (SABAH_IQ3S_FLOW=0: the phase-barrier kernel) agrees within TIGHT."""
    outs = []
    for flow in ("1", "0"):
        env = dict(os.environ, SABAH_IQ3S_FLOW=flow, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
        r = subprocess.run([sys.executable, "-c", _CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0, r.stderr[-3000:]
        outs.append(np.array([float(v) for v in r.stdout.strip().splitlines()[-1].split(",")]))
    from oracle import cpu as orc
    assert orc.rel_l2(outs[0], outs[1]) <= TIGHT


_CHILD = r"""
import ctypes, numpy as np, torch
from sabah_moe_accelerator_b200 import ops, rt
ops.init(0)
d_model, ff, E, K, n = 2048, 768, 64, 10, 3
banks = [tuple(ops.synth_rows(E * rows, k, 21, seed=4400 + 3 * L + r, sigma=0.02)
               for r, (rows, k) in enumerate(((ff, d_model), (ff, d_model), (d_model, ff)))) for L in range(n)]
rng = np.random.default_rng(44)
ids = torch.from_numpy(np.stack([rng.choice(E, K, replace=False) for _ in range(n)]).astype(np.int32)).cuda()
w = torch.full((n, K), 0.1, device="cuda")
x = torch.from_numpy(rng.standard_normal((1, d_model)).astype(np.float32)).cuda()
h = torch.empty((1, K, ff), device="cuda")
arr = ctypes.c_void_p * n
G, U, D = (arr(*[b[r].data_ptr() for b in banks]) for r in range(3))
gs, ds = ff * rt.row_bytes(21, d_model), d_model * rt.row_bytes(21, ff)
rt.check(rt.lib().sabah_moe_decode(n, G, U, D, gs, ds, E, ctypes.c_void_p(ids.data_ptr()),
         ctypes.c_void_p(w.data_ptr()), ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(h.data_ptr()), d_model, ff,
         K, 1, 21, 21, 21, ctypes.c_void_p(ops._stream(None))), "decode")
torch.cuda.synchronize()
print(",".join(repr(float(v)) for v in x.cpu().numpy()[0]))
"""


def test_bench_cfg2_token_all_layers(gpu_rt):
    """The benchmark's own workload: its 48-block x 512-expert bank (49.8 GB,
    bench.build_cfg2_bank) and its routing set 0, one token through all 48
    blocks, against the fp64 chain."""
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import bench
    st = torch.cuda.Stream()
    bank, views = bench.build_cfg2_bank(torch.device("cuda", 0), st, 0, bench.LAYERS)
    ids, w = bench.routing(1, bench.LAYERS)
    r = bench.cfg2_parity(views, ids[0], w[0], bench.x0())
    del views, bank
    torch.cuda.empty_cache()
    assert r <= TOL and r <= TIGHT, r


def test_flow_wait_that_never_ends_gives_up_and_recovers(gpu_rt):
    """Failure detection without a GPU fault: with the test switch
    SABAH_TEST_FLOW_STALL=1, one CTA first waits (short poll limit) for data
    that nothing writes. The kernel must give up instead of hanging: every CTA
    winds down, the device error word reads SB_DERR_TIMEOUT (2), and the next
    call, without the switch, is clean and bit-identical to a normal run."""
    d_model, ff, E, K, n_layers = 2048, 768, 64, 10, 3
    banks = _banks(n_layers, E, d_model, ff, seed=4500)
    rng = np.random.default_rng(45)
    ids, w = _routing(rng, n_layers, E, K)
    ids_d, w_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    x0 = torch.randn((1, d_model), device="cuda")
    h = torch.empty((1, K, ff), device="cuda")
    from sabah_moe_accelerator_b200 import rt
    x_ok = x0.clone()
    rt.check(_decode(gpu_rt, banks, ids_d, w_d, x_ok, h, d_model, ff, E), "sabah_moe_decode")
    torch.cuda.synchronize()
    os.environ["SABAH_TEST_FLOW_STALL"] = "1"
    try:
        x = x0.clone()
        rt.check(_decode(gpu_rt, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode (stalled)")
        torch.cuda.synchronize()   # returns: every wait is bounded
    finally:
        del os.environ["SABAH_TEST_FLOW_STALL"]
    assert gpu_rt.sabah_rt_device_error() == 2
    x = x0.clone()
    rt.check(_decode(gpu_rt, banks, ids_d, w_d, x, h, d_model, ff, E), "sabah_moe_decode after the timeout")
    torch.cuda.synchronize()
    assert gpu_rt.sabah_rt_device_error() == 0
    assert torch.equal(x, x_ok)
