"""Expert-parallel MoE bank over the GPUs of one node (one process per GPU).

Each rank holds, for every layer, the experts [e0, e1) with
owner(e) = floor(e * world / n_experts), and owns the tokens
[rank * T / world, (rank + 1) * T / world). One layer of a decode step:

1. all-gather the owned tokens' x              -> x_all [T][d_model]
2. gather the (token, slot) pairs whose expert is local (sorted by token,
   then slot)                                   -> xp [P][d_model]
3. the fused routed block on those pairs, one pair per "token", n_used = 1,
   with the pair's routing weight              -> yp [P][d_model] = w * Wd(silu(Wg x) * Wu x)
4. sum the pairs of each token in slot order   -> y [T][d_model]
5. reduce-scatter (sum over ranks)             -> y_own [T / world][d_model]
6. residual                                     x_own += y_own

Steps 1 and 5 are the exchange (NCCL all-gather and reduce-scatter over
NVLink); 2-4 and 6 run this package's kernels through the C ABI. Routing ids are
an input of MUL_MAT_ID (as in the reference's v2 contract, which downloads
them), so the pair plan is made on the host from host ids.

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


# ----------------------------------------------------------------- orchestration
def layer_step(x_own, plan_dev, layer, ops, comm):
    """One layer for this rank: x_own (T / world rows) <- x_own + block(x)."""
    x_all = comm.all_gather(x_own)
    P = plan_dev["n_pairs"]
    n_tok = x_all.shape[0]
    y = ops.empty_rows(n_tok)
    if P:
        yp = ops.empty_rows(P)
        if hasattr(ops, "block_rows"):   # the block reads the pairs' token rows in place
            ops.block_rows(layer, x_all, plan_dev["tok"], plan_dev["lid"], plan_dev["w"], yp)
        else:
            xp = ops.empty_rows(P)
            ops.gather(x_all, plan_dev["tok"], xp)
            ops.block(layer, xp, plan_dev["lid"], plan_dev["w"], yp)
        ops.sum_rows(yp, plan_dev["offsets"], y)
    else:
        ops.sum_rows(None, plan_dev["offsets"], y)
    y_own = comm.reduce_scatter(y)
    ops.add(x_own, y_own)
    return x_own


def decode_step(x_own, plans_dev, ops, comm):
    """All layers of one decode step; plans_dev[L] is layer L's device plan."""
    for L, pl in enumerate(plans_dev):
        layer_step(x_own, pl, L, ops, comm)
    return x_own


# ----------------------------------------------------------------- GPU side
class TorchComm:
    """NCCL (or any torch.distributed backend with these collectives)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)

    def all_gather(self, x_own):
        import torch
        out = torch.empty((x_own.shape[0] * self.world,) + tuple(x_own.shape[1:]), dtype=x_own.dtype,
                          device=x_own.device)
        self.dist.all_gather_into_tensor(out, x_own.contiguous(), group=self.group)
        return out

    def reduce_scatter(self, y):
        import torch
        out = torch.empty((y.shape[0] // self.world,) + tuple(y.shape[1:]), dtype=y.dtype, device=y.device)
        self.dist.reduce_scatter_tensor(out, y.contiguous(), group=self.group)
        return out


class SingleComm:
    """world = 1: the exchange is the identity."""

    def all_gather(self, x_own):
        return x_own

    def reduce_scatter(self, y):
        return y


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


def plan_to_device(plan: LayerPlan):
    """Host plan -> device tensors (int32 rows, [P][1] ids and weights)."""
    import torch
    return {"n_pairs": plan.n_pairs,
            "tok": torch.from_numpy(plan.tok).cuda(),
            "lid": torch.from_numpy(plan.lid.reshape(-1, 1)).cuda(),
            "w": torch.from_numpy(plan.w.reshape(-1, 1)).cuda(),
            "offsets": torch.from_numpy(plan.offsets).cuda()}
