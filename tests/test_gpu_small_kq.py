"""Q4_K / Q6_K fused block for 1-4 tokens (sabah_moe_block_ids through the
small-batch path: each distinct routed expert decoded once per block) against
the float64 reference_block (sabah/runtime/executor.py:134-159) over the same
bytes, dequantised as sb_host_dequant (sabah/runtime/cuda/sabah_rt.cu:2233-2423)
and gguf-py quants.py:586 (Q6_K)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-3
TIGHT = 2e-5
Q4_K, Q6_K = 12, 14


def _markov_ids(rng, T, K, E, p_keep=0.8):
    """Token 0 draws K distinct experts; each later token keeps the previous
    token's expert in a slot with p_keep, else draws a fresh one."""
    cur = rng.choice(E, K, replace=False)
    out = [cur.copy()]
    for _ in range(1, T):
        cur = cur.copy()
        for i in range(K):
            if rng.random() >= p_keep:
                while True:
                    e = int(rng.integers(E))
                    if e not in cur:
                        break
                cur[i] = e
        out.append(cur.copy())
    return np.stack(out).astype(np.int32)


def _banks(E, d_model, ff, qg, qd, seed):
    from sabah_moe_accelerator_b200 import ops
    gate = ops.synth_rows(E * ff, d_model, qg, seed=seed, sigma=0.02)
    up = ops.synth_rows(E * ff, d_model, qg, seed=seed + 1, sigma=0.02)
    down = ops.synth_rows(E * d_model, ff, qd, seed=seed + 2, sigma=0.02)
    return gate, up, down


def _want(orc, banks, E, ids, w, x, d_model, ff, qg, qd):
    g, u, d = (b.cpu().numpy().reshape(E, -1) for b in banks)
    return np.stack([orc.moe_block_f64(g, u, d, ids[t], w[t], x[t], d_model, ff, qg, qg, qd)
                     for t in range(ids.shape[0])])


@pytest.mark.parametrize("qg,qd,d_model,ff,T", [
    (Q4_K, Q6_K, 2048, 768, 1), (Q4_K, Q6_K, 2048, 768, 2), (Q4_K, Q6_K, 2048, 768, 3), (Q4_K, Q6_K, 2048, 768, 4),
    (Q6_K, Q4_K, 1024, 512, 4),    # Q6_K gate/up, Q4_K down copied row by row (288-byte rows)
    (Q4_K, Q4_K, 512, 2048, 2),    # down rows of 2048 (one expert per staged chunk)
])
def test_small_kq_block_matches_fp64(gpu_rt, orc, qg, qd, d_model, ff, T):
    from sabah_moe_accelerator_b200 import ops
    E, K = 32, 10
    banks = _banks(E, d_model, ff, qg, qd, seed=100 + d_model + T)
    rng = np.random.default_rng(7 * T + ff)
    ids = _markov_ids(rng, T, K, E)
    w = rng.random((T, K)).astype(np.float32) + 0.1
    w /= w.sum(1, keepdims=True)
    x = rng.standard_normal((T, d_model)).astype(np.float32)
    out = ops.moe_block_ids(*banks, torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(),
                            torch.from_numpy(x).cuda(), d_model, ff, E, qg, qg, qd)
    got = out.cpu().numpy()
    want = _want(orc, banks, E, ids, w, x, d_model, ff, qg, qd)
    for t in range(T):
        r = orc.rel_l2(got[t], want[t])
        assert r <= TOL and r <= TIGHT, (t, r)


def test_small_kq_duplicates_accumulate_and_determinism(gpu_rt, orc):
    """A token routed twice to one expert, all tokens sharing experts, a zero x
    row; accumulate adds to out; two runs agree bit for bit."""
    from sabah_moe_accelerator_b200 import ops
    d_model, ff, E, K, T = 2048, 768, 16, 10, 4
    banks = _banks(E, d_model, ff, Q4_K, Q6_K, seed=900)
    rng = np.random.default_rng(5)
    ids = np.stack([rng.permutation(E)[:K] for _ in range(T)]).astype(np.int32)
    ids[1, 7] = ids[1, 2]            # duplicate within token 1
    ids[3] = ids[0]                  # token 3 routes exactly as token 0
    w = (rng.random((T, K)) + 0.1).astype(np.float32)
    x = rng.standard_normal((T, d_model)).astype(np.float32)
    x[2] = 0.0
    ids_d, w_d, x_d = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda()
    a = ops.moe_block_ids(*banks, ids_d, w_d, x_d, d_model, ff, E, Q4_K, Q4_K, Q6_K)
    b = ops.moe_block_ids(*banks, ids_d, w_d, x_d, d_model, ff, E, Q4_K, Q4_K, Q6_K)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    got = a.cpu().numpy()
    assert float(np.abs(got[2]).max()) == 0.0
    want = _want(orc, banks, E, ids, w, x, d_model, ff, Q4_K, Q6_K)
    for t in (0, 1, 3):
        r = orc.rel_l2(got[t], want[t])
        assert r <= TOL and r <= TIGHT, (t, r)
    acc = x_d.clone()
    ops.moe_block_ids(*banks, ids_d, w_d, x_d, d_model, ff, E, Q4_K, Q4_K, Q6_K, out=acc, accumulate=True)
    torch.cuda.synchronize()
    assert orc.rel_l2(acc.cpu().numpy(), x + got) <= TIGHT


def test_small_kq_out_of_range_id(gpu_rt):
    from sabah_moe_accelerator_b200 import ops, rt
    d_model, ff, E, K, T = 2048, 768, 16, 10, 2
    banks = _banks(E, d_model, ff, Q4_K, Q6_K, seed=910)
    ids = np.tile(np.arange(K, dtype=np.int32), (T, 1))
    ids[1, 4] = E
    w = torch.full((T, K), 0.1, device="cuda")
    x = torch.randn(T, d_model, device="cuda")
    out = ops.moe_block_ids(*banks, torch.from_numpy(ids).cuda(), w, x, d_model, ff, E, Q4_K, Q4_K, Q6_K)
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    assert np.isnan(o[1]).all() and np.isfinite(o[0]).all()
    assert rt.lib().sabah_rt_device_error() == 1
