"""B200-native (sm_100a) routed-expert MUL_MAT_ID runtime.

A from-scratch implementation of the one hot operator of Sabah-MoE-Accelerator
behind its own C ABI (libsabah_rt.so): `sabah_rt_mul_mat_id_v2`, the fused
`sabah_moe_block`, and the helpers the reference's Python harness binds.
`rt` is the ctypes binding; `ops` wraps the calls for torch tensors.
"""
from . import rt  # noqa: F401

__all__ = ["rt"]
