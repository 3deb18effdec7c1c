"""sabah_dequant on the device: the kernels' own decoders, bit-exact against the
oracle (which is pinned to gguf-py and the reference), for all 11 types.
Reference: sabah/tests/test_quant_kernels.py (there rel < 1e-6; here bit-exact).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TYPES = {"Q5_1": 7, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ3_XXS": 18, "IQ4_NL": 20,
         "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "Q2_0": 42}


def _device_dequant(rtlib, raw: np.ndarray, qt: int, n_rows: int, row_elems: int) -> np.ndarray:
    d_src = torch.from_numpy(np.ascontiguousarray(raw).reshape(-1)).cuda()
    d_dst = torch.empty(n_rows * row_elems, dtype=torch.float32, device="cuda")
    from sabah_moe_accelerator_b200 import rt
    rt.check(rtlib.sabah_dequant(d_src.data_ptr(), d_dst.data_ptr(), qt, n_rows, row_elems), "dequant")
    return d_dst.cpu().numpy()


@pytest.mark.parametrize("name", sorted(TYPES))
def test_device_dequant_bit_exact_on_golden_blocks(gpu_rt, orc, golden, name):
    qt = TYPES[name]
    raw = golden["raw_" + name]
    be = orc.QBLOCK[qt][0]
    n = raw.shape[0] * be
    row = 256 if be <= 256 and n % 256 == 0 else n
    got = _device_dequant(gpu_rt, raw, qt, n // row, row)
    assert np.array_equal(got.view(np.uint32), orc.dequant(raw, qt, n).view(np.uint32))


@pytest.mark.parametrize("name", ["IQ3_S", "Q8_0", "Q4_K", "Q6_K"])
def test_synthetic_rows_decode_exactly_and_look_like_the_source(gpu_rt, orc, name):
    """The device encoder's bytes: device dequant == oracle dequant of the same
    bytes, and the decoded weights have the N(0, 0.02) shape they encode."""
    from sabah_moe_accelerator_b200 import ops, rt
    qt = TYPES[name]
    rows, k = 64, 2048
    raw = ops.synth_rows(rows, k, qt, seed=1234, sigma=0.02)
    torch.cuda.synchronize()
    host = raw.cpu().numpy()
    got = _device_dequant(gpu_rt, host, qt, rows, k)
    want = orc.dequant(host, qt, rows * k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.isfinite(want).all()
    assert 0.012 < float(want.std()) < 0.03, float(want.std())
    again = ops.synth_rows(rows, k, qt, seed=1234, sigma=0.02).cpu().numpy()
    assert np.array_equal(again, host), "synthetic bank is not reproducible"
    del rt
