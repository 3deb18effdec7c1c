// Internal launch interface between the C-ABI runtime (sb_runtime.cu) and the
// kernel translation units. Not part of the public ABI.
#pragma once

#include "sb_common.cuh"

#ifndef SABAH_SENTINEL
#define SABAH_SENTINEL 0
#endif

// Where the experts of one call live. Either a pointer table with one expert
// base per (token, slot) - the hot-tier path - or a device-resident bank that
// the kernel indexes with the router ids itself (no host round trip).
struct sb_experts {
    const void* const* ptrs;       // [n_tokens * n_ids] device pointers, or nullptr
    const uint8_t* base;           // bank base (used when ptrs == nullptr)
    size_t expert_stride;          // bytes between experts in the bank
    const int32_t* ids;            // router ids (used when ptrs == nullptr)
    size_t ids_id_stride;          // bytes
    size_t ids_token_stride;       // bytes
    int n_experts;
};

// One MUL_MAT_ID call, v2 byte-stride contract.
struct sb_mmid_args {
    sb_experts ex;
    size_t row_stride;
    const float* x;
    size_t x_id_stride;
    int x_rows;
    size_t x_token_stride;
    int n_ids, n_tokens;
    float* dst;
    size_t dst_id_stride, dst_token_stride;
    int rows, k, qt;
    int* err;                      // device-visible error word (host-mapped)
};

// One fused routed block over n_tokens tokens: gate/up + SwiGLU, then down +
// top-k weighted combine. Dense fp32 activations:
//   x [n_tokens][d_model], h [n_tokens][n_used][ff], out [n_tokens][d_model],
//   w [n_tokens][n_used] routing weights.
struct sb_block_args {
    sb_experts gate, up, down;
    const float* x;
    float* h;
    float* out;
    const float* w;
    int d_model, ff, n_used, n_tokens;
    int qt_gate, qt_up, qt_down;
    int accumulate;                // out += y instead of out = y
    int* err;
    const int32_t* xrows;          // optional: token t's input is row xrows[t] of x (nullptr: row t)
    int n_xrows;                   // rows of x when xrows is given
};

// device-side error codes written to *err
enum { SB_DERR_NONE = 0, SB_DERR_BAD_ID = 1, SB_DERR_TIMEOUT = 2, SB_DERR_MISALIGNED = 3 };

// Optional per-kernel timing (SABAH_LLAMA_EVENTS=1 or sabah_rt_kernel_timing):
// launches are bracketed by CUDA events on their own stream and accumulated
// per kernel name. sb_timing_begin returns a slot id (or -1 when off).
int sb_timing_begin(const char* name, cudaStream_t st);
void sb_timing_end(int slot, cudaStream_t st);

int sb_launch_mmid(const sb_mmid_args& a, cudaStream_t st);
int sb_launch_block(const sb_block_args& a, cudaStream_t st);
int sb_launch_dequant(const void* src, float* dst, int qt, int n_rows, int row_elems, cudaStream_t st);
bool sb_qt_supported(int qt);

// fast paths (sb_mmid_iq3s.cu); return 1 if the call was taken, 0 if the
// shape is not covered (caller falls back), -1 on a launch error
int sb_try_mmid_iq3s(const sb_mmid_args& a, cudaStream_t st);
// grouped tcgen05 path for many (token, slot) pairs on a device-resident bank
// (sb_prefill_iq3s.cu); same return convention
int sb_try_mmid_iq3s_grouped(const sb_mmid_args& a, cudaStream_t st, bool force = false);
// the fused block as grouped gate / up / down calls + SwiGLU + combine, for
// many (token, slot) pairs on device-resident banks; same return convention
int sb_block_iq3s_grouped(const sb_block_args& a, cudaStream_t st);
int sb_try_block_iq3s(const sb_block_args& a, cudaStream_t st);
// Q8_0 on the same tensor-core matvec engine (sb_mmid_iq3s.cu): MUL_MAT_ID,
// and the fused block as two launches; same return convention
int sb_try_mmid_q8_0(const sb_mmid_args& a, cudaStream_t st);
int sb_try_block_q8_0(const sb_block_args& a, cudaStream_t st);
// Q4_K / Q6_K fused block for 1-4 tokens on device banks, each distinct routed
// expert decoded once per block (sb_small_kq.cu): 1 taken, 0 not covered, -1 error
int sb_try_block_small(const sb_block_args& a, cudaStream_t st);
// sb_ep.cu: dst[i] = src[rows[i]]; indices outside [0, n_src) give NaN rows and
// SB_DERR_BAD_ID in *err (zero rows when err is null)
int sb_gather_rows(const float* src, int n_src, const int32_t* rows, int n, int k, float* dst, int* err,
                   cudaStream_t st);
// After a device error: the fused block's cross-CTA arrival counters may have
// been left mid-count by a kernel that gave up; the next call clears them.
void sb_block_scratch_invalidate();
// n_layers fused blocks of a decode step in one launch (sabah_moe_decode):
// x <- x + block_L(x) for L = 0..n_layers-1. Bank pointer arrays are host
// arrays of device pointers; ids / w are [n_layers][n_tokens][n_used].
struct sb_decode_args {
    int n_layers;
    const void* const* gate_banks;
    const void* const* up_banks;
    const void* const* down_banks;
    size_t gu_expert_stride, down_expert_stride;
    int n_experts;
    const int32_t* ids;
    const float* w;
    float* x;                // [n_tokens][d_model]: the input of block 0
    float* h;
    float* out;              // the last block's destination: out = (accumulate ? out : 0) + y; must be x
    int accumulate;          // when n_layers > 1 (the residual chain x += y)
    const int32_t* xrows;    // one block only, optional: token t's input is row xrows[t] of x
    int n_xrows;
    int d_model, ff, n_used, n_tokens;
    int qt_gate, qt_up, qt_down;
    int* err;
};
// persistent IQ3_S decode (sb_decode_iq3s.cu): 1 taken, 0 not covered, -1 error
int sb_try_decode_iq3s(const sb_decode_args& a, cudaStream_t st);
void sb_decode_scratch_invalidate();
// barrier-free persistent IQ3_S decode for one token (sb_flow_iq3s.cu), tried
// first by sb_try_decode_iq3s: 1 taken, 0 not covered, -1 error
int sb_try_flow_iq3s(const sb_decode_args& a, cudaStream_t st);
void sb_flow_scratch_invalidate();

// The IQ3_S fused block over a fixed device array instead of allocated scratch
// (sabah_moe_block_ids_noalloc); -1 with the error set when the call does not fit.
int sb_block_iq3s_fixed(const sb_block_args& a, cudaStream_t st);
