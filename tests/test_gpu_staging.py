"""Hot-tier fill paths of the host-source MUL_MAT_ID (the llama.cpp contract):
pageable memory and a file mapping go through the pinned staging ring (the
file by O_DIRECT reads where the file system allows them), pinned memory by
direct DMA (sabah/runtime/cuda/sabah_rt.cu:1033-1514, 2051-2116 in the
reference). Every case must be byte-exact in the slab (verified against the
source) and give the fp64 result.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

TOL = 2e-3
TIGHT = 2e-5


def _child(kind, tmp_path, env_extra=None):
    env = dict(os.environ, SABAH_LLAMA_HOT_BYTES=str(1 << 30), SABAH_LLAMA_VERIFY_BYTES="1")
    env.update(env_extra or {})
    code = _CHILD_LAYER if kind == "layer" else _CHILD
    r = subprocess.run([sys.executable, "-c", code, kind, str(tmp_path)], cwd=ROOT, env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("kind", ["pageable", "file", "pinned"])
def test_fill_sources_are_exact(tmp_path, kind):
    r = _child(kind, tmp_path)
    assert r["rel"] <= TOL and r["rel"] <= TIGHT, r
    s = r["snapshot"]
    assert s["verify_fail"] == 0 and s["verify_ok"] > 0, s
    assert s["misses"] > 0, s
    if kind == "pinned":
        assert s["pinned_fill_bytes"] > 0 and s["staged_bytes"] == 0, s
    else:
        assert s["staged_bytes"] >= s["bytes_fetched"] > 0 and s["pinned_fill_bytes"] == 0, s
        assert s["fill_waves"] >= 1, s
    if kind == "file":
        # O_DIRECT where the file system supports it; a fallback to the mapping otherwise
        assert s["direct_io_reads"] + s["direct_io_fallbacks"] > 0 or r["odirect_open"] is False, s
    if kind == "pageable":
        assert s["direct_io_reads"] == 0, s


def test_file_fill_without_direct_io(tmp_path):
    r = _child("file", tmp_path, {"SABAH_LLAMA_DIRECT_IO": "0"})
    assert r["rel"] <= TIGHT, r
    s = r["snapshot"]
    assert s["direct_io_reads"] == 0 and s["staged_bytes"] > 0 and s["verify_fail"] == 0, s


_CHILD = r"""
import json, os, sys
import numpy as np, torch
sys.path.insert(0, os.getcwd())
from oracle import cpu as orc
from sabah_moe_accelerator_b200 import ops, rt
kind, tmp = sys.argv[1], sys.argv[2]
ops.init(0)
qt, E, rows, k = 21, 64, 2048, 768       # IQ3_S down-shaped calls: one input row per slot
rb = rt.row_bytes(qt, k)
bank = ops.synth_rows(E * rows, k, qt, seed=123, sigma=0.02)
torch.cuda.synchronize()
host = bank.cpu().numpy()
odirect_open = None
if kind == "pageable":
    src = host.copy()
elif kind == "pinned":
    pin = torch.empty(host.size, dtype=torch.uint8).pin_memory()
    pin.numpy()[:] = host
    src = pin.numpy()
else:
    path = os.path.join(tmp, "bank.bin")
    host.tofile(path)
    src = np.memmap(path, dtype=np.uint8, mode="r")
    try:
        fd = os.open(path, os.O_RDONLY | os.O_DIRECT)
        os.close(fd)
        odirect_open = True
    except OSError:
        odirect_open = False
rng = np.random.default_rng(5)
T, K = 3, 10
ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
x = (rng.standard_normal((T, K, k)) * 0.1).astype(np.float32)
out = ops.mul_mat_id(src, rows * rb, rb, torch.from_numpy(x).cuda(), torch.from_numpy(ids).cuda(), rows, k, E, qt)
torch.cuda.synchronize()
exact = orc.mmid_f64(host, rows * rb, rb, x, K, ids, rows, k, E, qt)
print(json.dumps(dict(rel=orc.rel_l2(out.cpu().numpy(), exact), snapshot=rt.snapshot(), odirect_open=odirect_open)))
"""


def test_merged_layer_fetch_fills_followers_in_one_wave(tmp_path):
    """SABAH_LLAMA_LAYER_MERGE=1 (ref sabah_rt.cu:1944-2000): token 1 teaches
    the runtime the call chain gate -> up -> down with shared ids; on token 2
    the gate call's wave also fills the up and down experts, so the follower
    calls miss nothing. Every output stays exact and byte-verified."""
    r = _child("layer", tmp_path, {"SABAH_LLAMA_LAYER_MERGE": "1"})
    assert r["rel"] <= TIGHT, r
    s = r["snapshot"]
    assert s["verify_fail"] == 0 and s["verify_ok"] > 0, s
    assert r["merged_slots"] > 0, r
    assert r["follower_misses_token2"] == 0, r
    off = _child("layer", tmp_path, {"SABAH_LLAMA_LAYER_MERGE": "0"})
    assert off["rel"] <= TIGHT and off["merged_slots"] == 0 and off["follower_misses_token2"] > 0, off
    assert off["out_sha"] == r["out_sha"], "merged and per-call fetches gave different results"


def test_staging_readahead_serves_the_followers(tmp_path):
    """SABAH_LLAMA_PREFETCH=1 (ref sabah_rt.cu:1517-1860, 2051-2065): token 1
    teaches the runtime the call chain; on token 2 the gate call offers the up
    and down experts the tier lacks, reader threads read them from the file
    into pinned readahead buffers, and the follower calls' misses copy from
    there instead of reading the file again. Nothing is reserved in the tier:
    the followers still count their misses. Every output stays exact and
    byte-verified, and equal to the run without readahead."""
    r = _child("layer", tmp_path, {"SABAH_LLAMA_PREFETCH": "1", "SABAH_LLAMA_LAYER_MERGE": "0"})
    assert r["rel"] <= TIGHT, r
    s = r["snapshot"]
    assert s["verify_fail"] == 0 and s["verify_ok"] > 0, s
    assert s["prefetch_enabled"] == 1 and s["merged_slots"] == 0, s
    assert s["prefetch_reads"] > 0 and s["prefetch_used"] > 0, s
    assert s["prefetch_used_bytes"] <= s["prefetch_read_bytes"], s
    assert r["follower_misses_token2"] > 0, r
    off = _child("layer", tmp_path, {"SABAH_LLAMA_PREFETCH": "0", "SABAH_LLAMA_LAYER_MERGE": "0"})
    assert off["snapshot"]["prefetch_enabled"] == 0 and off["snapshot"]["prefetch_used"] == 0, off
    assert off["out_sha"] == r["out_sha"], "readahead and plain fetches gave different results"


_CHILD_LAYER = r"""
import hashlib, json, os, sys
import numpy as np, torch
sys.path.insert(0, os.getcwd())
from oracle import cpu as orc
from sabah_moe_accelerator_b200 import ops, rt
tmp = sys.argv[2]
ops.init(0)
qt, E, d_model, ff, K = 21, 32, 2048, 768, 10
rbg, rbd = rt.row_bytes(qt, d_model), rt.row_bytes(qt, ff)
parts = []
for seed, rows, k in ((31, ff, d_model), (32, ff, d_model), (33, d_model, ff)):
    t = ops.synth_rows(E * rows, k, qt, seed=seed, sigma=0.02)
    torch.cuda.synchronize()
    parts.append(t.cpu().numpy())
path = os.path.join(tmp, "layer.bin")
np.concatenate(parts).tofile(path)
m = np.memmap(path, dtype=np.uint8, mode="r")
gsz, dsz = parts[0].size, parts[2].size
g_src, u_src, d_src = m[:gsz], m[gsz:2 * gsz], m[2 * gsz:2 * gsz + dsz]
rng = np.random.default_rng(9)
outs, rels, follower_miss = [], [], None
for tok in range(2):
    ids = torch.from_numpy(rng.choice(E, K, replace=False).astype(np.int32)[None]).cuda()
    x = torch.from_numpy(rng.standard_normal((1, 1, d_model)).astype(np.float32)).cuda()
    key = ids.data_ptr()
    g = ops.mul_mat_id(g_src, ff * rbg, rbg, x, ids, ff, d_model, E, qt, ids_key=key)
    s0 = rt.snapshot()
    u = ops.mul_mat_id(u_src, ff * rbg, rbg, x, ids, ff, d_model, E, qt, ids_key=key)
    h = (torch.nn.functional.silu(g) * u).contiguous()
    dn = ops.mul_mat_id(d_src, d_model * rbd, rbd, h, ids, d_model, ff, E, qt, ids_key=key)
    torch.cuda.synchronize()
    s1 = rt.snapshot()
    if tok == 1:
        follower_miss = s1["misses"] - s0["misses"]
    ih, xh = ids.cpu().numpy(), x.cpu().numpy()
    wg = orc.mmid_f64(parts[0], ff * rbg, rbg, xh, 1, ih, ff, d_model, E, qt)
    wu = orc.mmid_f64(parts[1], ff * rbg, rbg, xh, 1, ih, ff, d_model, E, qt)
    wd = orc.mmid_f64(parts[2], d_model * rbd, rbd, h.cpu().numpy(), K, ih, d_model, ff, E, qt)
    for got, want in ((g, wg), (u, wu), (dn, wd)):
        rels.append(orc.rel_l2(got.cpu().numpy(), want))
    outs.append(dn.cpu().numpy())
snap = rt.snapshot()
print(json.dumps(dict(rel=max(rels), snapshot=snap, merged_slots=snap["merged_slots"],
                      follower_misses_token2=follower_miss,
                      out_sha=hashlib.sha256(np.concatenate([o.ravel() for o in outs]).tobytes()).hexdigest())))
"""
