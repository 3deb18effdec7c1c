"""Grouped IQ3_S MUL_MAT_ID (the tcgen05 prefill path, taken for >= 256
(token, slot) pairs on a device-resident bank) against the float64 recomputation
of sb_selfcheck (sabah/runtime/cuda/sabah_rt.cu:3435-3492) with the v2 row rule
x[t][i % x_rows] (sabah_rt.cu:3494-3515)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3     # rel-L2 per (token, slot) against fp64 (the contract)
TIGHT = 2e-5   # hi/lo fp16 operands, fp32 accumulation: ~1e-6 expected
QT = 21


def _check(got, want):
    for t in range(want.shape[0]):
        for i in range(want.shape[1]):
            w, g = want[t, i], got[t, i]
            r = float(np.linalg.norm(g - w) / max(np.linalg.norm(w), 1e-30))
            assert r <= TOL and r <= TIGHT, (t, i, r)


def _bank(E, rows, k, seed):
    from sabah_moe_accelerator_b200 import ops, rt
    rb = rt.row_bytes(QT, k)
    return ops.synth_rows(E * rows, k, QT, seed=seed, sigma=0.02), rb


@pytest.mark.parametrize("rows,k,x_rows", [(768, 2048, 1), (2048, 768, 10), (256, 1024, 1)])
def test_grouped_all_outputs_match_fp64(gpu_rt, orc, rows, k, x_rows):
    from sabah_moe_accelerator_b200 import ops
    E, K, T = 16, 10, 32                      # 320 pairs, ~20 per expert
    bank, rb = _bank(E, rows, k, seed=rows + k)
    rng = np.random.default_rng(rows)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    x = rng.standard_normal((T, x_rows, k)).astype(np.float32)
    out = ops.mul_mat_id(bank, rows * rb, rb, torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(),
                         rows, k, E, QT).cpu().numpy()
    want = orc.mmid_f64(bank.cpu().numpy(), rows * rb, rb, x, x_rows, ids, rows, k, E, QT)
    _check(out, want)


def test_grouped_expert_with_more_than_256_pairs(gpu_rt, orc):
    """Two experts, every token routed to both: 300 pairs each, split over two
    tasks per row tile."""
    from sabah_moe_accelerator_b200 import ops
    rows, k, E, K, T = 128, 512, 2, 2, 300
    bank, rb = _bank(E, rows, k, seed=77)
    rng = np.random.default_rng(3)
    ids = np.stack([rng.permutation(E) for _ in range(T)]).astype(np.int32)
    x = (rng.standard_normal((T, 1, k)) * np.exp(rng.uniform(-6, 6, (T, 1, 1)))).astype(np.float32)  # wide x range
    out = ops.mul_mat_id(bank, rows * rb, rb, torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(),
                         rows, k, E, QT).cpu().numpy()
    want = orc.mmid_f64(bank.cpu().numpy(), rows * rb, rb, x, 1, ids, rows, k, E, QT)
    _check(out, want)


def test_grouped_is_deterministic_and_handles_zero_rows(gpu_rt):
    from sabah_moe_accelerator_b200 import ops
    rows, k, E, K, T = 256, 768, 8, 8, 40
    bank, rb = _bank(E, rows, k, seed=9)
    rng = np.random.default_rng(9)
    ids = torch.from_numpy(np.stack([rng.permutation(E) for _ in range(T)]).astype(np.int32)).cuda()
    x = torch.from_numpy(rng.standard_normal((T, 1, k)).astype(np.float32)).cuda()
    x[5] = 0.0
    a = ops.mul_mat_id(bank, rows * rb, rb, x, ids, rows, k, E, QT)
    b = ops.mul_mat_id(bank, rows * rb, rb, x, ids, rows, k, E, QT)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert float(a[5].abs().max()) == 0.0
    assert torch.isfinite(a).all()


def test_grouped_out_of_range_id(gpu_rt):
    from sabah_moe_accelerator_b200 import ops, rt
    rows, k, E, K, T = 128, 256, 4, 4, 64
    bank, rb = _bank(E, rows, k, seed=4)
    ids = torch.from_numpy(np.tile(np.arange(K, dtype=np.int32), (T, 1))).cuda()
    ids[7, 2] = E
    x = torch.randn(T, 1, k, device="cuda")
    out = ops.mul_mat_id(bank, rows * rb, rb, x, ids, rows, k, E, QT)
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    assert np.isnan(o[7, 2]).all()
    o[7, 2] = 0.0
    assert np.isfinite(o).all()
    assert rt.lib().sabah_rt_device_error() == 1


@pytest.mark.parametrize("skew", [0.0, 1.2])
def test_grouped_light_and_mixed_experts(gpu_rt, orc, skew):
    """Many experts with few pairs each (the register-decode path: at most 8
    pairs per expert) and, with a Zipf-skewed routing, heavy experts beside
    them (the tcgen05 path) in one call."""
    from sabah_moe_accelerator_b200 import ops
    rows, k, E, K, T = 256, 1024, 64, 8, 40   # 320 pairs, 5 per expert on average
    bank, rb = _bank(E, rows, k, seed=int(skew * 10) + 5)
    rng = np.random.default_rng(17)
    p = 1.0 / np.arange(1, E + 1) ** skew
    p /= p.sum()
    ids = np.stack([rng.choice(E, K, replace=False, p=p) for _ in range(T)]).astype(np.int32)
    counts = np.bincount(ids.ravel(), minlength=E)
    light = int(((counts > 0) & (counts <= 8)).sum())
    assert light >= 40 and (skew == 0.0 or counts.max() > 8)
    x = rng.standard_normal((T, 1, k)).astype(np.float32)
    out = ops.mul_mat_id(bank, rows * rb, rb, torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(),
                         rows, k, E, QT).cpu().numpy()
    want = orc.mmid_f64(bank.cpu().numpy(), rows * rb, rb, x, 1, ids, rows, k, E, QT)
    _check(out, want)
