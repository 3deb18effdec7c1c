// Shared definitions for the sm_100a routed-expert runtime: ggml quant type
// codes, block geometry, error reporting.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>

// ggml type codes (ggml.h enum values; the reference keeps the same numbers at
// sabah/runtime/cuda/sabah_rt.cu:62-74, and Q6_K = 14 is added here).
enum sb_qtype : int {
    SB_Q5_1 = 7,
    SB_Q8_0 = 8,
    SB_Q4_K = 12,
    SB_Q5_K = 13,
    SB_Q6_K = 14,
    SB_IQ3_XXS = 18,
    SB_IQ4_NL = 20,
    SB_IQ3_S = 21,
    SB_IQ2_S = 22,
    SB_IQ4_XS = 23,
    SB_Q2_0 = 42,
};

// Elements and bytes per quant block (ggml-common.h block structs).
__host__ __device__ inline int sb_block_elems(int qt) {
    switch (qt) {
    case SB_Q5_1: case SB_Q8_0: case SB_IQ4_NL: return 32;
    case SB_Q2_0: return 64;
    case SB_Q4_K: case SB_Q5_K: case SB_Q6_K: case SB_IQ3_XXS:
    case SB_IQ3_S: case SB_IQ2_S: case SB_IQ4_XS: return 256;
    default: return 0;
    }
}

__host__ __device__ inline int sb_block_bytes(int qt) {
    switch (qt) {
    case SB_Q5_1: return 24;
    case SB_Q8_0: return 34;
    case SB_Q4_K: return 144;
    case SB_Q5_K: return 176;
    case SB_Q6_K: return 210;
    case SB_IQ3_XXS: return 98;
    case SB_IQ4_NL: return 18;
    case SB_IQ3_S: return 110;
    case SB_IQ2_S: return 82;
    case SB_IQ4_XS: return 136;
    case SB_Q2_0: return 18;
    default: return 0;
    }
}

// Bytes of one row of n elements (n a whole number of blocks), else 0.
__host__ __device__ inline size_t sb_row_bytes_of(int qt, long long n) {
    const int be = sb_block_elems(qt);
    if (be == 0 || n < 0 || n % be) return 0;
    return (size_t)(n / be) * (size_t)sb_block_bytes(qt);
}

// Error string shared by every entry point (last failure wins).
void sb_set_error(const char* fmt, ...);
bool sb_cuda_ok(cudaError_t e, const char* what);

#define SB_CUDA(call, what)                 \
    do {                                    \
        if (!sb_cuda_ok((call), (what))) {  \
            return -1;                      \
        }                                   \
    } while (0)
