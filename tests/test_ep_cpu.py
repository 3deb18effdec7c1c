"""Expert-parallel bank, host side (no GPU): the pair plan and the exchange.

The plan must partition every (token, slot) of a layer over the ranks exactly
once, in token-then-slot order. The layer data flow (all-gather, local pairs,
slot-ordered sum, reduce-scatter, residual) runs as world_size-2 gloo ranks with
a host stand-in for the kernels (the fp64 oracle block), and must reproduce
the single-process fp64 chain of reference_block (sabah/runtime/executor.py:134-159).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from sabah_moe_accelerator_b200 import ep

QT_Q8_0 = 8


def test_owner_and_ranges_are_consistent():
    for E in (8, 512, 13):
        for world in (1, 2, 3, 8):
            got = []
            for r in range(world):
                e0, e1 = ep.expert_range(r, E, world)
                got += list(range(e0, e1))
                assert all(ep.owner_of(e, E, world) == r for e in range(e0, e1))
            assert got == list(range(E))
    assert [ep.token_range(r, 64, 8) for r in range(8)][-1] == (56, 64)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_partitions_every_pair_once(world):
    rng = np.random.default_rng(world)
    T, K, E = 64, 10, 512
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, K)).astype(np.float32)
    seen = np.zeros((T, K), np.int32)
    for r in range(world):
        pl = ep.plan_layer(ids, w, r, world, E)
        e0, e1 = ep.expert_range(r, E, world)
        assert pl.offsets[0] == 0 and pl.offsets[-1] == pl.n_pairs
        assert np.all(np.diff(pl.offsets) >= 0)
        assert np.all(np.diff(pl.tok) >= 0)                 # sorted by token
        assert np.all((pl.lid >= 0) & (pl.lid < e1 - e0))
        for t in range(T):
            ks = [k for k in range(K) if e0 <= ids[t, k] < e1]   # slot order
            sl = slice(pl.offsets[t], pl.offsets[t + 1])
            assert list(pl.lid[sl] + e0) == [int(ids[t, k]) for k in ks]
            assert np.array_equal(pl.w[sl], w[t, ks])
            seen[t, ks] += 1
    assert np.all(seen == 1)


def test_plan_rejects_bad_ids():
    with pytest.raises(ValueError):
        ep.plan_layer(np.array([[0, 8]], np.int32), np.ones((1, 2), np.float32), 0, 2, 8)
    with pytest.raises(ValueError):
        ep.plan_layer(np.array([0, 1], np.int32), np.ones(2, np.float32), 0, 2, 8)


def test_empty_plan():
    pl = ep.plan_layer(np.array([[0, 1]], np.int32), np.ones((1, 2), np.float32), 1, 2, 8)
    assert pl.n_pairs == 0 and list(pl.offsets) == [0, 0]


# ------------------------------------------------------------- gloo data flow
D, F, E, K, T, LAYERS = 64, 64, 8, 2, 4, 2


def _q8_bank(rng, n_experts, rows, k):
    """n_experts x rows rows of k Q8_0 weights: fp16 scale + 32 int8 per block."""
    nb = n_experts * rows * (k // 32)
    blk = np.empty((nb, 34), np.uint8)
    blk[:, :2] = (rng.uniform(0.002, 0.02, nb).astype(np.float16)).view(np.uint8).reshape(nb, 2)
    blk[:, 2:] = rng.integers(-127, 128, (nb, 32)).astype(np.int8).view(np.uint8)
    return blk.reshape(n_experts, -1)


def _problem():
    rng = np.random.default_rng(11)
    banks = [(_q8_bank(rng, E, F, D), _q8_bank(rng, E, F, D), _q8_bank(rng, E, D, F)) for _ in range(LAYERS)]
    ids = np.stack([np.stack([rng.choice(E, K, replace=False) for _ in range(T)]) for _ in range(LAYERS)])
    w = rng.random((LAYERS, T, K)).astype(np.float32)
    x0 = rng.standard_normal((T, D)).astype(np.float64)
    return banks, ids.astype(np.int32), w, x0


class _HostOps:
    """Host stand-in for the kernels: the fp64 oracle block per pair."""

    def __init__(self, banks):
        from oracle import cpu
        self.cpu = cpu
        self.banks = banks

    def empty_rows(self, n):
        return np.zeros((n, D), np.float64)

    def gather(self, src, rows, dst):
        dst[:] = src[rows]

    def block(self, layer, xp, lid, w, out):
        g, u, d = self.banks[layer]
        for p in range(xp.shape[0]):
            out[p] = self.cpu.moe_block_f64(g, u, d, [int(lid[p, 0])], [float(w[p, 0])], xp[p].astype(np.float32),
                                            D, F, QT_Q8_0, QT_Q8_0, QT_Q8_0)

    def sum_rows_ex(self, src, n_src, idx, offsets, dst, init, init_row0):
        n_init = 0 if init is None else init.shape[0]
        for t in range(dst.shape[0]):
            acc = init[t - init_row0].copy() if init_row0 <= t < init_row0 + n_init else np.zeros(D)
            for i in range(offsets[t], offsets[t + 1]):
                r = i if idx is None else int(idx[i])
                if 0 <= r < n_src:
                    acc += src[r]
            dst[t] = acc


class _HostOpsRows(_HostOps):
    """The same stand-in with the gather folded into the block (ops.block_rows)."""

    def block_rows(self, layer, x_all, rows, lid, w, out):
        self.block(layer, x_all[rows], lid, w, out)


class _GlooComm:
    def __init__(self):
        import torch.distributed as dist
        self.dist = dist
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()

    def all_gather(self, x_own):
        import torch
        parts = [torch.empty(x_own.shape, dtype=torch.float64) for _ in range(self.world)]
        self.dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(x_own)))
        return torch.cat(parts).numpy()

    def reduce_scatter(self, y, out=None):
        import torch
        t = torch.from_numpy(np.ascontiguousarray(y))
        self.dist.all_reduce(t)
        n = y.shape[0] // self.world
        part = t.numpy()[self.rank * n:(self.rank + 1) * n]
        if out is None:
            return part.copy()
        out[:] = part
        return out

    def all_to_all(self, send, send_splits, recv, recv_splits):
        import torch
        r = torch.empty((recv.shape[0], D), dtype=torch.float64)
        self.dist.all_to_all_single(r, torch.from_numpy(np.ascontiguousarray(send)).reshape(-1, D),
                                    output_split_sizes=list(recv_splits), input_split_sizes=list(send_splits))
        recv[:] = r.numpy()
        return recv


def _rank_main(rank, world, port, out_path, rows_mode=False, exchange="ag"):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        banks, ids, w, x0 = _problem()
        e0, e1 = ep.expert_range(rank, E, world)
        local = [(g[e0:e1], u[e0:e1], d[e0:e1]) for g, u, d in banks]
        plans = []
        for L in range(LAYERS):
            if exchange == "ag":
                pl = ep.plan_layer(ids[L], w[L], rank, world, E)
                perm, pos = ep.expert_order(pl.lid)
                plans.append({"n_pairs": pl.n_pairs, "tok": pl.tok[perm], "lid": pl.lid[perm].reshape(-1, 1),
                              "w": pl.w[perm].reshape(-1, 1), "offsets": pl.offsets, "sum_idx": pos})
            else:
                pl = ep.plan_layer_a2a(ids[L], w[L], rank, world, E)
                perm, pos = ep.expert_order(pl.lid)
                plans.append({"n_pairs": pl.n_pairs, "n_send": sum(pl.send_splits), "n_recv": sum(pl.recv_splits),
                              "send_splits": pl.send_splits, "recv_splits": pl.recv_splits,
                              "send_rows": pl.send_rows, "pair_row": pl.pair_row[perm],
                              "lid": pl.lid[perm].reshape(-1, 1), "w": pl.w[perm].reshape(-1, 1),
                              "pair_off": pl.pair_off, "pair_sum_idx": pos, "comb_idx": pl.comb_idx,
                              "comb_off": pl.comb_off})
        t0, t1 = ep.token_range(rank, T, world)
        x_own = x0[t0:t1].copy()
        ops = _HostOpsRows(local) if rows_mode else _HostOps(local)
        ep.decode_step(x_own, plans, ops, _GlooComm(), exchange)
        np.save(out_path % rank, x_own)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("rows_mode,exchange,world", [(False, "ag", 2), (True, "ag", 2), (False, "a2a", 2),
                                                      (True, "a2a", 2), (True, "a2a", 4), (True, "ag", 4)])
def test_gloo_ranks_match_single_process_chain(tmp_path, orc, rows_mode, exchange, world):
    import torch.multiprocessing as mp
    out = str(tmp_path / "x_%d.npy")
    mp.start_processes(_rank_main, args=(world, _free_port(), out, rows_mode, exchange), nprocs=world,
                       start_method="spawn")
    got = np.concatenate([np.load(out % r) for r in range(world)])

    banks, ids, w, x0 = _problem()
    want = x0.copy()
    for L in range(LAYERS):
        g, u, d = banks[L]
        want = np.stack([want[t] + orc.moe_block_f64(g, u, d, ids[L, t], w[L, t], want[t].astype(np.float32), D, F,
                                                     QT_Q8_0, QT_Q8_0, QT_Q8_0) for t in range(T)])
    # fp64 sums in another order; x enters each block as fp32, as in the kernels
    assert orc.rel_l2(got, want) < 1e-6


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_a2a_plan_routes_every_pair_once(world):
    """The all-to-all plans of all ranks: every (token, slot) is computed on its
    expert's owner exactly once, on a row that carries that token, and every
    partial goes back to the token's owner exactly once per peer it visited."""
    rng = np.random.default_rng(100 + world)
    T_, K_, E_ = 64, 10, 512
    ids = np.stack([rng.choice(E_, K_, replace=False) for _ in range(T_)]).astype(np.int32)
    w = rng.random((T_, K_)).astype(np.float32)
    plans = [ep.plan_layer_a2a(ids, w, r, world, E_) for r in range(world)]
    seen = np.zeros((T_, K_), np.int32)
    for r, pl in enumerate(plans):
        assert sum(pl.send_splits) == pl.send_rows.size and sum(pl.recv_splits) == pl.pair_off.size - 1
        e0, e1 = ep.expert_range(r, E_, world)
        # the rows r receives, in the senders' order
        recv_tok = []
        for src in range(world):
            s0, _ = ep.token_range(src, T_, world)
            spl = plans[src].send_splits
            b = sum(spl[:r])
            recv_tok += list(s0 + plans[src].send_rows[b:b + spl[r]])
            assert spl[r] == pl.recv_splits[src]
        for j, t in enumerate(recv_tok):
            sl = slice(pl.pair_off[j], pl.pair_off[j + 1])
            assert np.all(pl.pair_row[sl] == j)
            ks = [k for k in range(K_) if e0 <= ids[t, k] < e1]
            assert list(pl.lid[sl] + e0) == [int(ids[t, k]) for k in ks] and np.array_equal(pl.w[sl], w[t, ks])
            seen[t, ks] += 1
        # combine: token i of r gets one partial from each peer that hosts one of its slots
        t0, t1 = ep.token_range(r, T_, world)
        for i in range(t1 - t0):
            got = pl.comb_idx[pl.comb_off[i]:pl.comb_off[i + 1]]
            peers = sorted({int(e) * world // E_ for e in ids[t0 + i]})
            assert len(got) == len(peers) and np.all(np.diff(got) > 0)
            base = np.concatenate([[0], np.cumsum(pl.send_splits)])
            for g_, d in zip(got, peers):
                assert base[d] <= g_ < base[d + 1] and pl.send_rows[g_] == i
    assert np.all(seen == 1)
