"""Child process for the MUL_MAT_ID contract cases that depend on environment
knobs read at sabah_rt_init (hot-tier size, byte verification, self-check) or
on which library is loaded (sentinel builds). Same pattern as the reference's
tests/test_mul_mat_id_contract.py:49-57: one v2 call with a HOST-backed expert
tensor, T=6 tokens, K=10 slots, ids drawn without replacement, x = N(0,1)*0.1.

Usage: python tests/mmid_child.py {down|gate} QT  -> one JSON line on stdout
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
sys.path.insert(0, ROOT)


def main(case: str, qt: int) -> dict:
    import torch
    from oracle import cpu as orc
    from sabah_moe_accelerator_b200 import ops, rt

    L = rt.lib()
    ops.init(0)
    E = 64
    if case == "down":
        rows, k = 2048, 768
    else:
        rows, k = 768, 2048
    rb = rt.row_bytes(qt, k)
    dev_bank = ops.synth_rows(E * rows, k, qt, seed=77 + qt, sigma=0.02)
    torch.cuda.synchronize()
    src = dev_bank.cpu().numpy()            # host-backed source: the llama.cpp contract
    rng = np.random.default_rng(4)
    T, K = 6, 10
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    x_rows = K if case == "down" else 1
    x = (rng.standard_normal((T, x_rows, k)) * 0.1).astype(np.float32)
    d_x, d_ids = torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda()
    out = ops.mul_mat_id(src, rows * rb, rb, d_x, d_ids, rows, k, E, qt, ids_key=d_ids.data_ptr())
    # second call on the same ids: hits only (and a reuse of the downloaded ids)
    out2 = ops.mul_mat_id(src, rows * rb, rb, d_x, d_ids, rows, k, E, qt, ids_key=d_ids.data_ptr())
    torch.cuda.synchronize()
    got, got2 = out.cpu().numpy(), out2.cpu().numpy()

    exact = orc.mmid_f64(src, rows * rb, rb, x, x_rows, ids, rows, k, E, qt)
    row0 = orc.mmid_f64(src, rows * rb, rb, np.ascontiguousarray(x[:, :1]), 1, ids, rows, k, E, qt)
    wrong = orc.mmid_f64(src, rows * rb, rb, x, x_rows, (ids + 1) % E, rows, k, E, qt)
    per_pair = [orc.rel_l2(got[t, i], exact[t, i]) for t in range(T) for i in range(K)]
    diag = [ctypes.c_ulonglong() for _ in range(5)]
    L.sabah_rt_get_diag(*[ctypes.byref(v) for v in diag])
    met = [ctypes.c_ulonglong() for _ in range(5)]
    L.sabah_rt_get_metrics(*[ctypes.byref(v) for v in met])
    return dict(case=case, qt=qt, rel_vs_exact=orc.rel_l2(got, exact), max_pair_rel=max(per_pair),
                maxabs_rel=float(np.abs(got - exact).max() / np.abs(exact).max()),
                repeat_identical=bool(np.array_equal(got, got2)),
                exact_vs_row0=orc.rel_l2(row0, exact) if x_rows > 1 else 0.0,
                rel_wrong_expert=orc.rel_l2(wrong, exact), out_sha=hashlib.sha256(got.tobytes()).hexdigest(),
                build_info=L.sabah_rt_build_info().decode(), snapshot=rt.snapshot(),
                calls=diag[0].value, tokens=diag[1].value, overflow=diag[2].value, verify_ok=diag[3].value,
                verify_fail=diag[4].value, hits=met[0].value, misses=met[1].value, evictions=met[2].value)


if __name__ == "__main__":
    print(json.dumps(main(sys.argv[1], int(sys.argv[2]))))
