"""Parity and speed against the reference's OWN CUDA path on the same bytes.

The reference runtime (sabah/runtime/cuda/sabah_rt.cu, compiled unmodified into
oracle/_ref/libsabah_rt_ref.so) runs in a child process (tests/ref_child.py):
its sabah_rt_mul_mat_id_v2 with a host source and TILE3 kernel (the default,
sabah_rt.cu:2929-3006), and its sabah_moe_block (k_gate_up / k_down,
:2725-2785) over a device pointer table. This build runs the same calls on the
same bytes. Both are checked against the fp64 oracle; this build must be at
least as close to it as the reference (or within TIGHT). The kernel-to-beat
test compares per-call device time at the decode shapes of the benchmark
configs: the reference's own CUDA-event timing (SABAH_LLAMA_EVENTS) against
this build's (sabah_rt_kernel_timing), kernels only, hot tier warm.
"""
from __future__ import annotations

import ctypes
import json
import os
import re
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

TOL = 2e-3
TIGHT = 2e-5
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libsabah_rt_ref.so")
GATE = (768, 2048)    # rows, k of a gate/up call at the benchmark shapes
DOWN = (2048, 768)


def _ref(mode, inputs, tmp_path, reps=0, env_extra=None):
    assert os.path.exists(REF_SO), "reference build missing (oracle/build_ref.sh): " + REF_SO
    inp, outp = str(tmp_path / ("in_%s.npz" % mode)), str(tmp_path / ("out_%s.npz" % mode))
    np.savez(inp, **inputs)
    env = dict(os.environ, SABAH_LLAMA_HOT_BYTES=str(4 << 30))
    env.pop("SABAH_RT_LIB", None)
    env.update(env_extra or {})
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "ref_child.py"), mode, inp, outp, str(reps)],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    d = np.load(outp)
    assert str(d["build_info"]).startswith("sabah_rt abi=v2"), str(d["build_info"])
    return d["out"], r.stderr


# Host sources stay alive for the whole module: the hot tier is keyed by the
# source address, as in the reference (a GGUF mapping lives as long as the
# process), so a freed array's address must not come back as a new tensor.
_SOURCES = []


def _case(qt, rows, k, E, T, n_ids, seed):
    from sabah_moe_accelerator_b200 import ops, rt
    bank = ops.synth_rows(E * rows, k, qt, seed=seed, sigma=0.02)
    torch.cuda.synchronize()
    src = bank.cpu().numpy().reshape(E, rows * rt.row_bytes(qt, k))
    _SOURCES.append(src)
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.choice(E, n_ids, replace=False) for _ in range(T)]).astype(np.int32)
    x_rows = n_ids if rows > k else 1    # down: one input row per slot; gate/up: broadcast
    x = rng.standard_normal((T, x_rows, k)).astype(np.float32)
    return src, ids, x


def _ours_mmid(src, ids, x, rows, k, E, qt, reps=0):
    from sabah_moe_accelerator_b200 import ops, rt
    rb = rt.row_bytes(qt, k)
    d_x, d_ids = torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda()
    out = None
    for _ in range(reps + 1):
        out = ops.mul_mat_id(src, rows * rb, rb, d_x, d_ids, rows, k, E, qt)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("qt,shape", [(21, GATE), (21, DOWN), (8, GATE), (8, DOWN), (12, GATE)])
def test_mmid_matches_reference_cuda_path(gpu_rt, orc, tmp_path, qt, shape):
    from sabah_moe_accelerator_b200 import rt
    rows, k = shape
    E, T, n_ids = 64, 2, 10
    src, ids, x = _case(qt, rows, k, E, T, n_ids, seed=70 + qt + rows)
    ref, _ = _ref("mmid", dict(source=src, x=x, ids=ids, rows=rows, k=k, E=E, qt=qt), tmp_path)
    ours = _ours_mmid(src, ids, x, rows, k, E, qt)
    rb = rt.row_bytes(qt, k)
    exact = orc.mmid_f64(src.reshape(-1), rows * rb, rb, x, x.shape[1], ids, rows, k, E, qt)
    r_ref, r_ours = orc.rel_l2(ref, exact), orc.rel_l2(ours, exact)
    assert r_ref <= TOL, ("reference vs fp64", r_ref)
    assert r_ours <= TOL and r_ours <= max(r_ref, TIGHT), ("ours vs fp64", r_ours, "reference", r_ref)
    assert orc.rel_l2(ours, ref) <= TOL


@pytest.mark.parametrize("qt", [21, 8])
def test_block_matches_reference_cuda_path(gpu_rt, orc, tmp_path, qt):
    from sabah_moe_accelerator_b200 import ops, rt
    d_model, ff, E, K = 2048, 768, 64, 10
    g = ops.synth_rows(E * ff, d_model, qt, seed=81, sigma=0.02)
    u = ops.synth_rows(E * ff, d_model, qt, seed=82, sigma=0.02)
    d = ops.synth_rows(E * d_model, ff, qt, seed=83, sigma=0.02)
    torch.cuda.synchronize()
    gh, uh, dh = (t.cpu().numpy().reshape(E, -1) for t in (g, u, d))
    rng = np.random.default_rng(84)
    ids = rng.choice(E, K, replace=False).astype(np.int32)
    w = rng.random(K).astype(np.float32)
    w /= w.sum()
    x = rng.standard_normal(d_model).astype(np.float32)
    ref, _ = _ref("block", dict(gate=gh, up=uh, down=dh, ids=ids, w=w, x=x, d_model=d_model, ff=ff,
                                qts=np.array([qt, qt, qt])), tmp_path)
    # this build, the same ABI call over the same kind of pointer table
    gs, ds = gh.shape[1], dh.shape[1]
    ptrs = torch.tensor([g.data_ptr() + int(e) * gs for e in ids] + [u.data_ptr() + int(e) * gs for e in ids] +
                        [d.data_ptr() + int(e) * ds for e in ids], dtype=torch.int64, device="cuda")
    d_x, d_w = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    out, h = torch.zeros(d_model, device="cuda"), torch.empty((K, ff), device="cuda")
    rt.check(rt.lib().sabah_moe_block(ctypes.c_void_p(d_x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                      ctypes.c_void_p(h.data_ptr()), ctypes.c_void_p(ptrs.data_ptr()),
                                      ctypes.c_void_p(d_w.data_ptr()), d_model, ff, K, qt, qt, qt, 0),
             "sabah_moe_block")
    torch.cuda.synchronize()
    ours = out.cpu().numpy()
    exact = orc.moe_block_f64(gh, uh, dh, ids, w, x, d_model, ff, qt, qt, qt)
    r_ref, r_ours = orc.rel_l2(ref, exact), orc.rel_l2(ours, exact)
    assert r_ref <= TOL, ("reference vs fp64", r_ref)
    assert r_ours <= TOL and r_ours <= max(r_ref, TIGHT), ("ours vs fp64", r_ours, "reference", r_ref)


def _ours_per_call_us(src, ids, x, rows, k, E, qt, reps):
    from sabah_moe_accelerator_b200 import rt
    L = rt.lib()
    _ours_mmid(src, ids, x, rows, k, E, qt)          # fills the hot tier
    L.sabah_rt_kernel_timing(1)
    _ours_mmid(src, ids, x, rows, k, E, qt, reps=reps - 1)
    buf = ctypes.create_string_buffer(8192)
    L.sabah_rt_kernel_times(buf, 8192)
    L.sabah_rt_kernel_timing(0)
    times = json.loads(buf.value.decode())
    return 1e3 * sum(v[1] for v in times.values()) / reps, times


@pytest.mark.parametrize("qt,shape,name", [(21, GATE, "cfg2 gate/up call"), (21, DOWN, "cfg2 down call"),
                                           (8, GATE, "cfg1 gate/up call"), (8, DOWN, "cfg1 down call")])
def test_kernel_to_beat(gpu_rt, tmp_path, qt, shape, name):
    """Per-call device time of one decode-token MUL_MAT_ID call (T = 1, top-10
    of 512 experts) against the reference's default TILE3 kernel on the same
    bytes; hot tier warm on both sides."""
    rows, k = shape
    E, reps = 512, 50
    src, ids, x = _case(qt, rows, k, E, 1, 10, seed=90 + qt + rows)
    _, err = _ref("mmid", dict(source=src, x=x, ids=ids, rows=rows, k=k, E=E, qt=qt), tmp_path, reps=reps,
                  env_extra={"SABAH_LLAMA_EVENTS": "1", "SABAH_LLAMA_TRACE": "1"})
    m = re.search(r"SABAH_EV .*?tile3=(\d).*?\| gu calls=(\d+) kernel_ms=[\d.]+ per_token=[\d.]+ per_call_us=([\d.]+)"
                  r" \| dn calls=(\d+) kernel_ms=[\d.]+ per_token=[\d.]+ per_call_us=([\d.]+)", err)
    assert m, err[-2000:]
    assert m.group(1) == "1", "the reference ran without TILE3"
    ref_us = float(m.group(3)) if rows < 1024 else float(m.group(5))
    assert int(m.group(2) if rows < 1024 else m.group(4)) >= reps
    ours_us, times = _ours_per_call_us(src, ids, x, rows, k, E, qt, reps)
    print("KERNEL_TO_BEAT %s qt=%d rows=%d k=%d: reference TILE3 %.2f us/call, this build %.2f us/call (%s)"
          % (name, qt, rows, k, ref_us, ours_us, ", ".join(times)))
    assert ours_us < ref_us, (name, ours_us, ref_us)
