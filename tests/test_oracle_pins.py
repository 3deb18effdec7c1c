"""The CPU oracle is pinned before it is trusted (CPU only).

Pins, per quant type, on the committed golden blocks:
  * gguf-py's dequantize (the reference harness's own dequant oracle,
    sabah/tests/test_quant_kernels.py:84-89) - bit-exact;
  * the reference's own sabah_rt_host_dequant, compiled from its sources
    (oracle/build_ref.sh) - bit-exact (the reference contract test
    tests/test_mul_mat_id_contract.py:101-109 demands max_abs_diff == 0);
  * small MUL_MAT_ID and fused-block cases computed with gguf-py + numpy float64.
"""
from __future__ import annotations

import numpy as np
import pytest

TYPES = {"Q5_1": 7, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ3_XXS": 18, "IQ4_NL": 20,
         "IQ3_S": 21, "IQ2_S": 22, "IQ4_XS": 23, "Q2_0": 42}


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", sorted(TYPES))
def test_oracle_dequant_matches_golden_bit_exactly(orc, golden, name):
    raw = golden["raw_" + name]
    qt = TYPES[name]
    n = raw.shape[0] * orc.QBLOCK[qt][0]
    got = orc.dequant(raw, qt, n)
    pinned = 0
    for side in ("gguf_", "ref_"):
        if side + name in golden:
            assert np.array_equal(_bits(got), _bits(golden[side + name])), side + name
            pinned += 1
    assert pinned >= 1, "type %s has no pin" % name


@pytest.mark.parametrize("name", sorted(TYPES))
def test_oracle_dequant_matches_live_gguf_py(orc, name):
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as Q
    if not hasattr(Q, name):
        pytest.skip("gguf-py has no %s" % name)
    qt = TYPES[name]
    be, bb = orc.QBLOCK[qt]
    rng = np.random.default_rng(qt)
    raw = rng.integers(0, 256, size=(200, bb), dtype=np.uint8)
    for off in {"Q5_1": [0, 2], "Q4_K": [0, 2], "Q5_K": [0, 2], "Q6_K": [208]}.get(name, [0]):
        raw[:, off:off + 2] = (rng.standard_normal(200) * 0.05).astype(np.float16).view(np.uint8).reshape(200, 2)
    want = np.asarray(quants.dequantize(raw, getattr(Q, name)), np.float32).reshape(-1)
    got = orc.dequant(raw, qt, 200 * be)
    assert np.array_equal(_bits(got), _bits(want))


def test_oracle_dequant_matches_reference_build_live(orc):
    if not orc.ref_available():
        pytest.skip("reference build absent (oracle/build_ref.sh)")
    rng = np.random.default_rng(7)
    for name, qt in TYPES.items():
        be, bb = orc.QBLOCK[qt]
        raw = rng.integers(0, 256, size=(64, bb), dtype=np.uint8)
        for off in {"Q5_1": [0, 2], "Q4_K": [0, 2], "Q5_K": [0, 2], "Q6_K": [208]}.get(name, [0]):
            raw[:, off:off + 2] = (rng.standard_normal(64)).astype(np.float16).view(np.uint8).reshape(64, 2)
        ref = orc.ref_dequant(raw, qt, 64 * be)
        if ref is None:
            assert name == "Q6_K", "reference unexpectedly lacks %s" % name
            continue
        assert np.array_equal(_bits(orc.dequant(raw, qt, 64 * be)), _bits(ref)), name


def test_oracle_rejects_partial_blocks_and_unknown_types(orc):
    import ctypes
    raw = np.zeros(110, np.uint8)
    out = np.empty(256, np.float32)
    assert orc.lib().orc_dequant(raw.ctypes.data, out.ctypes.data, 21, 100) == -1
    assert orc.lib().orc_dequant(raw.ctypes.data, out.ctypes.data, 99, 256) == -1
    del ctypes


@pytest.mark.parametrize("name", ["IQ3_S", "Q8_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("mode", ["bcast", "perslot"])
def test_oracle_mmid_matches_golden(orc, golden, name, mode):
    p = "mmid_%s_%s_" % (name, mode)
    src, ids, x, want = golden[p + "src"], golden[p + "ids"], golden[p + "x"], golden[p + "want"]
    qt = TYPES[name]
    E = src.shape[0]
    rows, k = want.shape[2], x.shape[2]
    rb = orc.row_bytes(qt, k)
    got = orc.mmid_f64(src, rows * rb, rb, x, x.shape[1], ids, rows, k, E, qt)
    np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-12)


def test_oracle_mmid_rejects_out_of_range_id(orc, golden):
    p = "mmid_IQ3_S_bcast_"
    src, ids, x = golden[p + "src"], golden[p + "ids"].copy(), golden[p + "x"]
    ids[1, 2] = src.shape[0]
    rb = orc.row_bytes(21, 512)
    with pytest.raises(ValueError):
        orc.mmid_f64(src, 8 * rb, rb, x, 1, ids, 8, 512, src.shape[0], 21)


@pytest.mark.parametrize("bname", ["iq3s", "q4k_q6k"])
def test_oracle_block_matches_golden(orc, golden, bname):
    p = "block_%s_" % bname
    qg, qu, qd = [int(v) for v in golden[p + "types"]]
    want = golden[p + "want"]
    got = orc.moe_block_f64(golden[p + "gate"], golden[p + "up"], golden[p + "down"], golden[p + "ids"],
                            golden[p + "w"], golden[p + "x"], want.shape[0], 256, qg, qu, qd)
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)


def test_cpu_baseline_decode_agrees_with_fp64_block(orc, golden):
    """The timed fp32 CPU baseline computes the same block (one layer)."""
    p = "block_iq3s_"
    gate, up, down = golden[p + "gate"], golden[p + "up"], golden[p + "down"]
    d_model, ff = 256, 256
    gs, ds = gate.shape[1], down.shape[1]
    x = golden[p + "x"]
    y = orc.decode_f32([gate.ctypes.data], [up.ctypes.data], [down.ctypes.data], gs, ds, 21, 21,
                       golden[p + "ids"][None, :], golden[p + "w"][None, :], x, d_model, ff, 3)
    want = x.astype(np.float64) + golden[p + "want"]
    assert orc.rel_l2(y, want) < 1e-5
