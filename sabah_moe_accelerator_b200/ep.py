"""Expert-parallel MoE bank over the GPUs of one node (one process per GPU).

Each rank holds, for every layer, the experts [e0, e1) with
owner(e) = floor(e * world / n_experts), and owns the tokens
[rank * T / world, (rank + 1) * T / world) (T divisible by world). A layer of a
decode step runs with one of two exchanges:

all-gather + reduce-scatter ("ag"):
1. all-gather the owned tokens' x                     -> x_all [T][d_model]
2. the fused routed block on the (token, slot) pairs whose expert is local
   (sorted by token, then slot), reading each pair's token row of x_all in
   place, one pair per "token", n_used = 1, with the pair's weight
                                                       -> yp [P][d_model]
3. per token, in slot order, the pairs' sum, plus x on the owned rows
                                                       -> y [T][d_model]
4. reduce-scatter (sum over ranks) straight into x_own: x_own = x + sum of y

all-to-all dispatch + combine ("a2a"):
1. dispatch: each rank sends every peer (itself included, rank order) the
   owned token rows that have a slot on that peer's experts; per-peer row
   counts come from the plan                          -> recv [R][d_model]
2. the block on the local pairs of the received rows  -> yp [P][d_model]
3. per received row, the sum of its pairs in slot order -> part [R][d_model]
4. combine: the partial rows go back to their tokens' owners (the reverse
   all-to-all)                                          -> back [S][d_model]
5. x_own[t] = x_own[t] + the partials of t in peer (rank) order

The collectives are NCCL over NVLink (torch.distributed). The kernels are this
package's (C ABI): sabah_moe_block_gather and sabah_ep_sum_rows_ex, which
folds the residual into the pair sums. Routing ids are an input of MUL_MAT_ID,
as in the reference's v2 contract, which downloads them. So the plans of a
step (all layers) are made on the host from host ids and go to the GPU as one
packed buffer.

The orchestration takes its compute and collective operations as objects so
the same data flow runs on GPUs (CudaOps + TorchComm over NCCL) and in the CPU
tests (gloo + a host stand-in).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import rt


def owner_of(expert: int, n_experts: int, world: int) -> int:
    return expert * world // n_experts


def expert_range(rank: int, n_experts: int, world: int) -> tuple[int, int]:
    """[e0, e1): the experts whose owner is `rank`."""
    e0 = -(-rank * n_experts // world)
    e1 = -(-(rank + 1) * n_experts // world)
    return e0, e1


def token_range(rank: int, n_tokens: int, world: int) -> tuple[int, int]:
    return rank * n_tokens // world, (rank + 1) * n_tokens // world


@dataclass
class LayerPlan:
    """This rank's (token, slot) pairs of one layer, sorted by token then slot."""
    tok: np.ndarray       # [P] int32 token of each pair
    lid: np.ndarray       # [P] int32 local expert id (expert - e0)
    w: np.ndarray         # [P] float32 routing weight
    offsets: np.ndarray   # [T + 1] int32: pairs of token t are offsets[t] .. offsets[t+1] - 1

    @property
    def n_pairs(self) -> int:
        return int(self.tok.shape[0])


def plan_layer(ids: np.ndarray, w: np.ndarray, rank: int, world: int, n_experts: int) -> LayerPlan:
    """Pairs of one layer routed to experts of `rank`. ids, w: [T][n_used]."""
    ids = np.asarray(ids)
    w = np.asarray(w, np.float32)
    if ids.ndim != 2 or ids.shape != w.shape:
        raise ValueError("ids and w must both be [n_tokens][n_used]")
    if ids.size and (ids.min() < 0 or ids.max() >= n_experts):
        raise ValueError("expert id outside [0, n_experts)")
    e0, e1 = expert_range(rank, n_experts, world)
    mask = (ids >= e0) & (ids < e1)
    t_idx, k_idx = np.nonzero(mask)            # row-major: sorted by token, then slot
    counts = mask.sum(1)
    offsets = np.zeros(ids.shape[0] + 1, np.int32)
    np.cumsum(counts, out=offsets[1:])
    return LayerPlan(tok=t_idx.astype(np.int32), lid=(ids[t_idx, k_idx] - e0).astype(np.int32),
                     w=w[t_idx, k_idx].astype(np.float32), offsets=offsets)


@dataclass
class A2APlan:
    """This rank's side of one layer's all-to-all exchange (host arrays).

    send_rows / send_splits: owned token rows (relative to the first owned
    token) sent to each peer in rank order, token order within a peer.
    recv_splits: rows received from each peer; received row j is a token of
    that peer, token order within the peer.
    pair_row / lid / w / pair_off: the local pairs, sorted by received row,
    then slot; pair_off[j] .. pair_off[j+1] - 1 are the pairs of received
    row j.
    comb_idx / comb_off: for owned token i, the rows of the combine buffer
    (which mirrors send_rows) holding its partials, in peer order."""
    send_rows: np.ndarray
    send_splits: list
    recv_splits: list
    pair_row: np.ndarray
    lid: np.ndarray
    w: np.ndarray
    pair_off: np.ndarray
    comb_idx: np.ndarray
    comb_off: np.ndarray

    @property
    def n_pairs(self) -> int:
        return int(self.pair_row.shape[0])


def plan_layer_a2a(ids: np.ndarray, w: np.ndarray, rank: int, world: int, n_experts: int) -> A2APlan:
    """The all-to-all plan of one layer for `rank`. ids, w: [T][n_used], the
    layer's routing for all T tokens (every rank plans from the same ids)."""
    ids = np.asarray(ids)
    w = np.asarray(w, np.float32)
    if ids.ndim != 2 or ids.shape != w.shape:
        raise ValueError("ids and w must both be [n_tokens][n_used]")
    if ids.size and (ids.min() < 0 or ids.max() >= n_experts):
        raise ValueError("expert id outside [0, n_experts)")
    T = ids.shape[0]
    if T % world:
        raise ValueError("the token count must be a multiple of the world size")
    owner = (ids.astype(np.int64) * world) // n_experts          # [T][K] owner rank of each slot
    hits = np.zeros((world, T), bool)                             # [world][T]: token t has a slot on d
    hits[owner, np.arange(T)[:, None]] = True
    t0, t1 = token_range(rank, T, world)
    # dispatch: owned tokens needed by each peer, peer by peer, token order within
    own = hits[:, t0:t1]
    send_splits = own.sum(1).astype(np.int64).tolist()
    send_rows = np.nonzero(own)[1].astype(np.int32)
    # receive: every token with a slot here, in token order, which is peer order
    recv_tok = np.nonzero(hits[rank])[0]
    recv_splits = np.bincount(recv_tok // (T // world), minlength=world).astype(np.int64).tolist()
    mine = owner[recv_tok] == rank                                # [R][K]
    j_idx, k_idx = np.nonzero(mine)                               # by received row, then slot
    pair_off = np.zeros(recv_tok.size + 1, np.int32)
    np.cumsum(mine.sum(1), out=pair_off[1:])
    e0, _ = expert_range(rank, n_experts, world)
    toks = recv_tok[j_idx]
    # combine: owned token i's partials sit in the combine buffer at the rows
    # where send_rows put it, peer by peer (row of (d, i) = start of peer d's
    # block + rank of i among the tokens sent to d)
    base = np.concatenate([[0], np.cumsum(send_splits)])[:world].astype(np.int64)
    row_of = base[:, None] + np.cumsum(own, axis=1) - 1
    mask_t = own.T                                                # [n_own][world], peer order per token
    comb_idx = row_of.T[mask_t].astype(np.int32)
    comb_off = np.zeros(t1 - t0 + 1, np.int32)
    np.cumsum(mask_t.sum(1), out=comb_off[1:])
    return A2APlan(send_rows=send_rows, send_splits=send_splits, recv_splits=recv_splits, pair_row=j_idx.astype(np.int32),
                   lid=(ids[toks, k_idx] - e0).astype(np.int32), w=w[toks, k_idx].astype(np.float32),
                   pair_off=pair_off, comb_idx=comb_idx, comb_off=comb_off)


def expert_order(lid: np.ndarray):
    """(perm, pos): the pairs in expert order (stable, so token / row order
    within an expert) for the block, where pairs of one expert run back to
    back and re-read its tiles from L2; pos[i] = where pair i (in plan order)
    sits in that order, the index list of the slot-ordered sums."""
    perm = np.argsort(np.asarray(lid).reshape(-1), kind="stable").astype(np.int32)
    pos = np.empty_like(perm)
    pos[perm] = np.arange(perm.size, dtype=np.int32)
    return perm, pos


# ----------------------------------------------------------------- orchestration
def layer_step(x_own, plan_dev, layer, ops, comm):
    """One layer, all-gather arm: x_own (T / world rows) <- x_own + block(x)."""
    x_all = comm.all_gather(x_own)
    P = plan_dev["n_pairs"]
    n_tok, n_own = x_all.shape[0], x_own.shape[0]
    yp = None
    if P:
        yp = ops.empty_rows(P)
        if hasattr(ops, "block_rows"):   # the block reads the pairs' token rows in place
            ops.block_rows(layer, x_all, plan_dev["tok"], plan_dev["lid"], plan_dev["w"], yp)
        else:
            xp = ops.empty_rows(P)
            ops.gather(x_all, plan_dev["tok"], xp)
            ops.block(layer, xp, plan_dev["lid"], plan_dev["w"], yp)
    idx = plan_dev.get("sum_idx")   # pairs computed in expert order, summed in slot order
    if comm.world == 1:
        # the sums land in x itself: x = x + pairs
        ops.sum_rows_ex(yp, P, idx, plan_dev["offsets"], x_own, x_own, 0)
        return x_own
    y = ops.empty_rows(n_tok)
    ops.sum_rows_ex(yp, P, idx, plan_dev["offsets"], y, x_own, comm.rank * n_own)
    comm.reduce_scatter(y, out=x_own)
    return x_own


def layer_step_a2a(x_own, plan_dev, layer, ops, comm):
    """One layer, all-to-all arm: dispatch the token rows each peer needs,
    the local pairs, combine the partials back at their tokens' owners."""
    n_send, n_recv, P = plan_dev["n_send"], plan_dev["n_recv"], plan_dev["n_pairs"]
    send = ops.empty_rows(n_send)
    ops.gather(x_own, plan_dev["send_rows"], send)
    recv = ops.empty_rows(n_recv)
    comm.all_to_all(send, plan_dev["send_splits"], recv, plan_dev["recv_splits"])
    part = ops.empty_rows(n_recv)
    yp = None
    if P:
        yp = ops.empty_rows(P)
        if hasattr(ops, "block_rows"):
            ops.block_rows(layer, recv, plan_dev["pair_row"], plan_dev["lid"], plan_dev["w"], yp)
        else:
            xp = ops.empty_rows(P)
            ops.gather(recv, plan_dev["pair_row"], xp)
            ops.block(layer, xp, plan_dev["lid"], plan_dev["w"], yp)
    ops.sum_rows_ex(yp, P, plan_dev.get("pair_sum_idx"), plan_dev["pair_off"], part, None, 0)
    back = ops.empty_rows(n_send)
    comm.all_to_all(part, plan_dev["recv_splits"], back, plan_dev["send_splits"])
    ops.sum_rows_ex(back, n_send, plan_dev["comb_idx"], plan_dev["comb_off"], x_own, x_own, 0)
    return x_own


def decode_step(x_own, plans_dev, ops, comm, exchange: str = "ag"):
    """All layers of one decode step; plans_dev[L] is layer L's device plan
    (plan_to_device / pack_plans for "ag", pack_plans_a2a for "a2a")."""
    step = layer_step if exchange == "ag" else layer_step_a2a
    for L, pl in enumerate(plans_dev):
        step(x_own, pl, L, ops, comm)
    return x_own


# ----------------------------------------------------------------- GPU side
class TorchComm:
    """NCCL (or any torch.distributed backend with these collectives)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, x_own):
        import torch
        out = torch.empty((x_own.shape[0] * self.world,) + tuple(x_own.shape[1:]), dtype=x_own.dtype,
                          device=x_own.device)
        self.dist.all_gather_into_tensor(out, x_own.contiguous(), group=self.group)
        return out

    def reduce_scatter(self, y, out=None):
        import torch
        if out is None:
            out = torch.empty((y.shape[0] // self.world,) + tuple(y.shape[1:]), dtype=y.dtype, device=y.device)
        self.dist.reduce_scatter_tensor(out, y.contiguous(), group=self.group)
        return out

    def all_to_all(self, send, send_splits, recv, recv_splits):
        self.dist.all_to_all_single(recv, send, output_split_sizes=list(recv_splits),
                                    input_split_sizes=list(send_splits), group=self.group)
        return recv


class SingleComm:
    """world = 1: the exchange is the identity."""
    world, rank = 1, 0

    def all_gather(self, x_own):
        return x_own

    def reduce_scatter(self, y, out=None):
        if out is not None and out is not y:
            out.copy_(y)
            return out
        return y

    def all_to_all(self, send, send_splits, recv, recv_splits):
        recv.copy_(send)
        return recv


class CudaOps:
    """This package's kernels through the C ABI, on torch device tensors."""

    def __init__(self, banks, d_model: int, ff: int, n_local_experts: int, qt: int, stream=None):
        """banks[L] = (gate, up, down) local expert tensors of layer L (uint8, device)."""
        import torch
        self.torch = torch
        self.banks = banks
        self.d_model, self.ff, self.E = d_model, ff, n_local_experts
        self.qt = qt
        self.gs = ff * rt.row_bytes(qt, d_model)
        self.ds = d_model * rt.row_bytes(qt, ff)
        self.L = rt.lib()
        self.stream = stream
        self._h = None

    def _st(self):
        s = self.stream if self.stream is not None else self.torch.cuda.current_stream()
        return ctypes.c_void_p(s.cuda_stream or 1)

    def empty_rows(self, n):
        return self.torch.empty((n, self.d_model), dtype=self.torch.float32, device="cuda")

    def gather(self, src, rows, dst):
        rt.check(self.L.sabah_ep_gather_rows(ctypes.c_void_p(src.data_ptr()), src.shape[0],
                                             ctypes.c_void_p(rows.data_ptr()), dst.shape[0], self.d_model,
                                             ctypes.c_void_p(dst.data_ptr()), self._st()), "sabah_ep_gather_rows")

    def block(self, layer, xp, lid, w, out):
        P = xp.shape[0]
        if self._h is None or self._h.shape[0] < P:
            self._h = self.torch.empty((P, 1, self.ff), dtype=self.torch.float32, device="cuda")
        g, u, d = self.banks[layer]
        rt.check(self.L.sabah_moe_block_ids(ctypes.c_void_p(g.data_ptr()), ctypes.c_void_p(u.data_ptr()),
                                            ctypes.c_void_p(d.data_ptr()), self.gs, self.ds, self.E,
                                            ctypes.c_void_p(lid.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                            ctypes.c_void_p(xp.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                            ctypes.c_void_p(self._h.data_ptr()), self.d_model, self.ff, 1, P,
                                            self.qt, self.qt, self.qt, 0, self._st()), "sabah_moe_block_ids")

    def block_rows(self, layer, x_all, rows, lid, w, out):
        """The block on rows `rows` of x_all (one per pair), without a gather pass."""
        P = out.shape[0]
        if self._h is None or self._h.shape[0] < P:
            self._h = self.torch.empty((P, 1, self.ff), dtype=self.torch.float32, device="cuda")
        g, u, d = self.banks[layer]
        rt.check(self.L.sabah_moe_block_gather(ctypes.c_void_p(g.data_ptr()), ctypes.c_void_p(u.data_ptr()),
                                               ctypes.c_void_p(d.data_ptr()), self.gs, self.ds, self.E,
                                               ctypes.c_void_p(lid.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                                               ctypes.c_void_p(x_all.data_ptr()), ctypes.c_void_p(rows.data_ptr()),
                                               x_all.shape[0], ctypes.c_void_p(out.data_ptr()),
                                               ctypes.c_void_p(self._h.data_ptr()), self.d_model, self.ff, 1, P,
                                               self.qt, self.qt, self.qt, 0, self._st()), "sabah_moe_block_gather")

    def sum_rows(self, src, offsets, dst):
        n_src = 0 if src is None else src.shape[0]
        ptr = ctypes.c_void_p(src.data_ptr() if src is not None else dst.data_ptr())
        rt.check(self.L.sabah_ep_sum_rows(ptr, n_src, ctypes.c_void_p(offsets.data_ptr()), dst.shape[0],
                                          self.d_model, ctypes.c_void_p(dst.data_ptr()), self._st()),
                 "sabah_ep_sum_rows")

    def add(self, x, y):
        rt.check(self.L.sabah_ep_add(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), x.numel(),
                                     self._st()), "sabah_ep_add")

    def sum_rows_ex(self, src, n_src, idx, offsets, dst, init, init_row0):
        """dst[t] = init rows (from init_row0) + the src rows of t (sabah_ep_sum_rows_ex)."""
        vp = lambda t: ctypes.c_void_p(t.data_ptr() if t is not None else 0)
        n_init = 0 if init is None else init.shape[0]
        rt.check(self.L.sabah_ep_sum_rows_ex(vp(src), n_src if src is not None else 0, vp(idx), vp(offsets),
                                             dst.shape[0], self.d_model, vp(dst), vp(init), init_row0, n_init,
                                             self._st()), "sabah_ep_sum_rows_ex")


def plan_to_device(plan: LayerPlan):
    """Host plan -> device tensors (int32 rows, [P][1] ids and weights)."""
    import torch
    return {"n_pairs": plan.n_pairs,
            "tok": torch.from_numpy(plan.tok).cuda(),
            "lid": torch.from_numpy(plan.lid.reshape(-1, 1)).cuda(),
            "w": torch.from_numpy(plan.w.reshape(-1, 1)).cuda(),
            "offsets": torch.from_numpy(plan.offsets).cuda()}


def _pack(arrays, device):
    """int32 / float32 host arrays -> one device int32 buffer (one pinned
    upload), returned as device views in the same order."""
    import torch
    sizes = [int(a.size) for a in arrays]
    host = torch.empty(max(1, sum(sizes)), dtype=torch.int32, pin_memory=True)
    hv = host.numpy()
    o = 0
    for a, n in zip(arrays, sizes):
        hv[o:o + n] = np.ascontiguousarray(a).reshape(-1).view(np.int32)
        o += n
    dev = host.to(device, non_blocking=True)
    views, o = [], 0
    for a, n in zip(arrays, sizes):
        v = dev[o:o + n]
        views.append(v.view(torch.float32) if a.dtype == np.float32 else v)
        o += n
    return views, host   # the pinned buffer lives as long as the upload may be in flight


def pack_plans(plans, device="cuda"):
    """All-gather plans of a step (one per layer) -> device plans in one upload."""
    arrays = []
    for pl in plans:
        perm, pos = expert_order(pl.lid)
        arrays += [pl.tok[perm], pl.lid[perm], pl.w[perm], pl.offsets, pos]
    views, keep = _pack(arrays, device)
    out = []
    for i, pl in enumerate(plans):
        tok, lid, w, off, pos = views[5 * i:5 * i + 5]
        out.append({"n_pairs": pl.n_pairs, "tok": tok, "lid": lid.view(-1, 1), "w": w.view(-1, 1),
                    "offsets": off, "sum_idx": pos, "_keep": keep})
    return out


def pack_plans_a2a(plans, device="cuda"):
    """All-to-all plans of a step -> device plans in one upload."""
    arrays = []
    for pl in plans:
        perm, pos = expert_order(pl.lid)
        arrays += [pl.send_rows, pl.pair_row[perm], pl.lid[perm], pl.w[perm], pl.pair_off, pos, pl.comb_idx,
                   pl.comb_off]
    views, keep = _pack(arrays, device)
    out = []
    for i, pl in enumerate(plans):
        send_rows, pair_row, lid, w, pair_off, pos, comb_idx, comb_off = views[8 * i:8 * i + 8]
        out.append({"n_pairs": pl.n_pairs, "n_send": int(sum(pl.send_splits)), "n_recv": int(sum(pl.recv_splits)),
                    "send_splits": pl.send_splits, "recv_splits": pl.recv_splits, "send_rows": send_rows,
                    "pair_row": pair_row, "lid": lid.view(-1, 1), "w": w.view(-1, 1), "pair_off": pair_off,
                    "pair_sum_idx": pos, "comb_idx": comb_idx, "comb_off": comb_off, "_keep": keep})
    return out
