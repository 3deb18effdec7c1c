"""PyTorch-facing wrappers over the C ABI.

torch provides device memory and the current stream; every computation runs in
libsabah_rt.so. Tensors are passed by data_ptr(), streams by cuda_stream.
"""
from __future__ import annotations

import ctypes

import torch

from . import rt

_initialised_device = None


def init(device: int = 0) -> None:
    """sabah_rt_init once per process (re-initialising resets the hot tier)."""
    global _initialised_device
    if _initialised_device is None:
        torch.cuda.set_device(device)
        rt.check(rt.lib().sabah_rt_init(device), "sabah_rt_init")
        _initialised_device = device


def _stream(stream) -> int:
    """Raw stream handle for the C ABI. torch's default stream has handle 0,
    which the ABI reads as "the runtime's own stream"; it is passed as the
    explicit legacy-stream handle (cudaStreamLegacy = 1) instead."""
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or 1


def _ptr(t) -> int:
    if isinstance(t, torch.Tensor):
        return t.data_ptr()
    return int(t.ctypes.data)   # numpy array (host-backed source)


def row_bytes(qt: int, k: int) -> int:
    return rt.row_bytes(qt, k)


def synth_rows(n_rows: int, k: int, qt: int, seed: int, sigma: float = 0.02, out: torch.Tensor | None = None,
               stream=None) -> torch.Tensor:
    """n_rows dense rows of k elements of type qt encoding N(0, sigma) weights."""
    nbytes = n_rows * rt.row_bytes(qt, k)
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    assert out.numel() >= nbytes and out.is_cuda
    rt.check(rt.lib().sabah_synth_rows(ctypes.c_void_p(out.data_ptr()), qt, n_rows, k, seed, sigma,
                                       ctypes.c_void_p(_stream(stream))), "synth_rows")
    return out


def mul_mat_id(source, expert_stride: int, row_stride: int, x: torch.Tensor, ids: torch.Tensor, rows: int,
               k: int, n_experts: int, qt: int, out: torch.Tensor | None = None, stream=None, ids_key=None):
    """MUL_MAT_ID through sabah_rt_mul_mat_id_v2 on dense tensors.

    source: the expert tensor (a CUDA uint8 tensor = resident bank, or a host
    numpy array = the hot-tier path). x: [T, x_rows, k] float32, ids: [T, n_ids]
    int32, out: [T, n_ids, rows] float32.
    """
    T, n_ids = ids.shape
    x_rows = x.shape[1]
    assert x.shape == (T, x_rows, k) and x.dtype == torch.float32 and x.is_contiguous()
    assert ids.dtype == torch.int32 and ids.is_contiguous()
    if out is None:
        out = torch.empty((T, n_ids, rows), dtype=torch.float32, device="cuda")
    rc = rt.mul_mat_id_v2(_ptr(source), expert_stride, row_stride, x.data_ptr(), k * 4, x_rows, x_rows * k * 4,
                          ids.data_ptr(), 4, n_ids * 4, n_ids, T, out.data_ptr(), rows * 4, n_ids * rows * 4,
                          rows, k, n_experts, qt, _stream(stream), ids_key)
    rt.check(rc, "sabah_rt_mul_mat_id_v2")
    return out


def moe_block_ids(gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, ids: torch.Tensor, w: torch.Tensor,
                  x: torch.Tensor, d_model: int, ff: int, n_experts: int, qt_gate: int, qt_up: int, qt_down: int,
                  out: torch.Tensor | None = None, h: torch.Tensor | None = None, accumulate: bool = False,
                  stream=None) -> torch.Tensor:
    """Fused routed block on device-resident banks: out (+)= sum_e w * Wd (silu(Wg x) * Wu x)."""
    T, n_used = ids.shape
    if out is None:
        out = torch.empty((T, d_model), dtype=torch.float32, device="cuda")
    if h is None:
        h = torch.empty((T, n_used, ff), dtype=torch.float32, device="cuda")
    gs = ff * rt.row_bytes(qt_gate, d_model)
    ds = d_model * rt.row_bytes(qt_down, ff)
    assert rt.row_bytes(qt_up, d_model) == rt.row_bytes(qt_gate, d_model)
    L = rt.lib()
    rc = L.sabah_moe_block_ids(ctypes.c_void_p(gate.data_ptr()), ctypes.c_void_p(up.data_ptr()),
                               ctypes.c_void_p(down.data_ptr()), gs, ds, n_experts,
                               ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(w.data_ptr()),
                               ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                               ctypes.c_void_p(h.data_ptr()), d_model, ff, n_used, T, qt_gate, qt_up, qt_down,
                               1 if accumulate else 0, ctypes.c_void_p(_stream(stream)))
    rt.check(rc, "sabah_moe_block_ids")
    return out
