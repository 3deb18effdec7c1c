// Per-type decoders for the ggml expert quant formats.
//
// Every format is handled in units of 32 elements ("sub-block s" of a row).
// A decoder turns sub-block s into
//     q[l]  small signed integers (exact in fp32 and fp16), l = 0..31
//     S0/S1 the scale of elements 0..15 / 16..31
//     O     an additive offset (only Q5_1, Q4_K, Q5_K have one)
// so that the dequantized element is  fl(fl(S * q) + O)  - the exact rounding
// sequence of gguf-py's dequantize_blocks for that type, which is also the
// sequence of the reference's host dequantizer (sabah_rt.cu:2233-2423). The
// dequant entry points use that form and are bit-exact; the matvec kernels use
// the same decode but the algebraically equal  S0*sum(q x) + S1*sum(q x) + O*sum(x).
//
// Block layouts (byte offsets) follow ggml-common.h:
//   Q8_0  34: d | qs[32] int8
//   Q5_1  24: d | m | qh u32 | qs[16]
//   Q4_K 144: d | dmin | scales[12] | qs[128]
//   Q5_K 176: d | dmin | scales[12] | qh[32] | qs[128]
//   Q6_K 210: ql[128] | qh[64] | scales[16] int8 | d
//   IQ3_XXS 98: d | qs[64] | 8 x u32 (four 7-bit sign indices + 4-bit scale)
//   IQ4_NL 18: d | qs[16]
//   IQ3_S 110: d | qs[64] | qh[8] | signs[32] | scales[4]
//   IQ2_S  82: d | qs[32] | signs[32] | qh[8] | scales[8]
//   IQ4_XS 136: d | scales_h u16 | scales_l[4] | qs[128]
//   Q2_0  18: d | qs[16] (2-bit codes, 64 elements)
#pragma once

#include "sb_common.cuh"
#include "sb_tables.h"

#include <type_traits>

// sb_tables.h (generated) holds every table twice: sb_<name> in device memory
// for the kernels and sb_h_<name> in host memory for the host dequantizer.
__host__ __device__ inline uint32_t sb_t_iq3s(int i) {
#ifdef __CUDA_ARCH__
    return sb_iq3s_grid[i];
#else
    return sb_h_iq3s_grid[i];
#endif
}
__host__ __device__ inline uint32_t sb_t_iq3xxs(int i) {
#ifdef __CUDA_ARCH__
    return sb_iq3xxs_grid[i];
#else
    return sb_h_iq3xxs_grid[i];
#endif
}
__host__ __device__ inline uint64_t sb_t_iq2s(int i) {
#ifdef __CUDA_ARCH__
    return sb_iq2s_grid[i];
#else
    return sb_h_iq2s_grid[i];
#endif
}
__host__ __device__ inline int sb_t_ksigns(int i) {
#ifdef __CUDA_ARCH__
    return sb_ksigns[i];
#else
    return sb_h_ksigns[i];
#endif
}
__host__ __device__ inline int sb_t_kv4(int i) {
#ifdef __CUDA_ARCH__
    return sb_kvalues_iq4nl[i];
#else
    return sb_h_kvalues_iq4nl[i];
#endif
}

// binary16 bits at p (little endian, 2-byte aligned or not) -> float, exact
__host__ __device__ inline float sb_f16(const uint8_t* p) {
    const unsigned short bits = (unsigned short)(p[0] | (p[1] << 8));
#ifdef __CUDA_ARCH__
    return __half2float(__ushort_as_half(bits));
#else
    __half_raw r;
    r.x = bits;
    return __half2float(__half(r));
#endif
}

__host__ __device__ inline uint32_t sb_u32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// rounding-exact float ops (no FMA contraction on either side)
__host__ __device__ inline float sb_mul(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    volatile float r = a * b;
    return r;
#endif
}
__host__ __device__ inline float sb_add(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fadd_rn(a, b);
#else
    volatile float r = a + b;
    return r;
#endif
}

// 6-bit (scale, min) pair j of the 12-byte K-quant scale field
__host__ __device__ inline void sb_kscale(const uint8_t* sc, int j, int& s, int& m) {
    if (j < 4) {
        s = sc[j] & 63;
        m = sc[j + 4] & 63;
    } else {
        s = (sc[j + 4] & 15) | ((sc[j - 4] >> 6) << 4);
        m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

struct sb_sub {
    int q[32];
    float s0, s1, off;
    bool has_off;
};

// Decode sub-block s (32 elements) of a row of type QT into u.
template <int QT>
__host__ __device__ inline void sb_decode(const uint8_t* row, int s, sb_sub& u) {
    u.has_off = false;
    u.off = 0.f;
    if constexpr (QT == SB_Q8_0) {
        const uint8_t* b = row + (size_t)s * 34;
        u.s0 = u.s1 = sb_f16(b);
#pragma unroll
        for (int l = 0; l < 32; ++l) u.q[l] = (int8_t)b[2 + l];
    } else if constexpr (QT == SB_Q5_1) {
        const uint8_t* b = row + (size_t)s * 24;
        u.s0 = u.s1 = sb_f16(b);
        u.off = sb_f16(b + 2);
        u.has_off = true;
        const uint32_t qh = sb_u32(b + 4);
#pragma unroll
        for (int l = 0; l < 16; ++l) {
            u.q[l] = (b[8 + l] & 15) | (int)(((qh >> l) & 1u) << 4);
            u.q[l + 16] = (b[8 + l] >> 4) | (int)(((qh >> (l + 16)) & 1u) << 4);
        }
    } else if constexpr (QT == SB_Q4_K || QT == SB_Q5_K) {
        const int j = s & 7;
        const uint8_t* b = row + (size_t)(s >> 3) * (QT == SB_Q4_K ? 144 : 176);
        int sc, mn;
        sb_kscale(b + 4, j, sc, mn);
        u.s0 = u.s1 = sb_mul(sb_f16(b), (float)sc);
        u.off = -sb_mul(sb_f16(b + 2), (float)mn);
        u.has_off = true;
        const uint8_t* q = b + (QT == SB_Q4_K ? 16 : 48) + (j >> 1) * 32;
        const int sh = (j & 1) * 4;
#pragma unroll
        for (int l = 0; l < 32; ++l) {
            int v = (q[l] >> sh) & 15;
            if constexpr (QT == SB_Q5_K) v |= ((b[16 + l] >> j) & 1) << 4;
            u.q[l] = v;
        }
    } else if constexpr (QT == SB_Q6_K) {
        const int j = s & 7;
        const uint8_t* b = row + (size_t)(s >> 3) * 210;
        const int h = j >> 2, p = j & 3;
        const float d = sb_f16(b + 208);
        const int8_t* sc = (const int8_t*)(b + 192);
        u.s0 = sb_mul(d, (float)sc[2 * j]);
        u.s1 = sb_mul(d, (float)sc[2 * j + 1]);
        const uint8_t* ql = b + 64 * h + (p & 1) * 32;
        const uint8_t* qh = b + 128 + 32 * h;
        const int lsh = (p >> 1) * 4, hsh = 2 * p;
#pragma unroll
        for (int l = 0; l < 32; ++l)
            u.q[l] = (((ql[l] >> lsh) & 15) | (((qh[l] >> hsh) & 3) << 4)) - 32;
    } else if constexpr (QT == SB_IQ3_XXS) {
        const int j = s & 7;
        const uint8_t* b = row + (size_t)(s >> 3) * 98;
        const uint32_t a = sb_u32(b + 66 + 4 * j);
        u.s0 = u.s1 = sb_mul(sb_mul(sb_f16(b), sb_add(0.5f, (float)(a >> 28))), 0.5f);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int sg = sb_t_ksigns((a >> (7 * g)) & 127);
            const uint32_t w0 = sb_t_iq3xxs(b[2 + 8 * j + 2 * g]);
            const uint32_t w1 = sb_t_iq3xxs(b[2 + 8 * j + 2 * g + 1]);
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int v0 = (w0 >> (8 * m)) & 255, v1 = (w1 >> (8 * m)) & 255;
                u.q[8 * g + m] = (sg >> m) & 1 ? -v0 : v0;
                u.q[8 * g + 4 + m] = (sg >> (m + 4)) & 1 ? -v1 : v1;
            }
        }
    } else if constexpr (QT == SB_IQ4_NL) {
        const uint8_t* b = row + (size_t)s * 18;
        u.s0 = u.s1 = sb_f16(b);
#pragma unroll
        for (int l = 0; l < 16; ++l) {
            u.q[l] = sb_t_kv4(b[2 + l] & 15);
            u.q[l + 16] = sb_t_kv4(b[2 + l] >> 4);
        }
    } else if constexpr (QT == SB_IQ3_S) {
        const int j = s & 7;
        const uint8_t* b = row + (size_t)(s >> 3) * 110;
        const int nib = (b[106 + (j >> 1)] >> (4 * (j & 1))) & 15;
        u.s0 = u.s1 = sb_mul(sb_f16(b), (float)(1 + 2 * nib));
        const int qh = b[66 + j];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int sg = b[74 + 4 * j + g];
            const uint32_t w0 = sb_t_iq3s(b[2 + 8 * j + 2 * g] | (((qh >> (2 * g)) & 1) << 8));
            const uint32_t w1 = sb_t_iq3s(b[2 + 8 * j + 2 * g + 1] | (((qh >> (2 * g + 1)) & 1) << 8));
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int v0 = (w0 >> (8 * m)) & 255, v1 = (w1 >> (8 * m)) & 255;
                u.q[8 * g + m] = (sg >> m) & 1 ? -v0 : v0;
                u.q[8 * g + 4 + m] = (sg >> (m + 4)) & 1 ? -v1 : v1;
            }
        }
    } else if constexpr (QT == SB_IQ2_S) {
        const int j = s & 7;
        const uint8_t* b = row + (size_t)(s >> 3) * 82;
        const int sc = b[74 + j];
        const float d = sb_f16(b);
        u.s0 = sb_mul(sb_mul(d, sb_add(0.5f, (float)(sc & 15))), 0.25f);
        u.s1 = sb_mul(sb_mul(d, sb_add(0.5f, (float)(sc >> 4))), 0.25f);
        const int qh = b[66 + j];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint64_t w = sb_t_iq2s(b[2 + 4 * j + g] | (((qh >> (2 * g)) & 3) << 8));
            const int sg = b[34 + 4 * j + g];
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int v = (int)((w >> (8 * m)) & 255);
                u.q[8 * g + m] = (sg >> m) & 1 ? -v : v;
            }
        }
    } else if constexpr (QT == SB_IQ4_XS) {
        const int j = s & 7;
        const uint8_t* b = row + (size_t)(s >> 3) * 136;
        const int sh = b[2] | (b[3] << 8);
        const int ls = ((b[4 + (j >> 1)] >> (4 * (j & 1))) & 15) | (((sh >> (2 * j)) & 3) << 4);
        u.s0 = u.s1 = sb_mul(sb_f16(b), (float)(ls - 32));
        const uint8_t* q = b + 8 + 16 * j;
#pragma unroll
        for (int l = 0; l < 16; ++l) {
            u.q[l] = sb_t_kv4(q[l] & 15);
            u.q[l + 16] = sb_t_kv4(q[l] >> 4);
        }
    } else if constexpr (QT == SB_Q2_0) {
        const uint8_t* b = row + (size_t)(s >> 1) * 18;
        u.s0 = u.s1 = sb_f16(b);
        const uint8_t* q = b + 2 + (s & 1) * 8;
#pragma unroll
        for (int l = 0; l < 32; ++l) u.q[l] = ((q[l >> 2] >> (2 * (l & 3))) & 3) - 1;
    }
}

// Dequantize sub-block s into y[0..31], bit-exact against gguf-py.
template <int QT>
__host__ __device__ inline void sb_dequant32(const uint8_t* row, int s, float* y) {
    sb_sub u;
    sb_decode<QT>(row, s, u);
#pragma unroll
    for (int l = 0; l < 32; ++l) {
        const float v = sb_mul(l < 16 ? u.s0 : u.s1, (float)u.q[l]);
        y[l] = u.has_off ? sb_add(v, u.off) : v;
    }
}

// fp32 dot of sub-block s with x[0..31] (generic matvec path).
template <int QT>
__device__ inline float sb_dot32(const uint8_t* row, int s, const float* x) {
    sb_sub u;
    sb_decode<QT>(row, s, u);
    float a0 = 0.f, a1 = 0.f, sx = 0.f;
#pragma unroll
    for (int l = 0; l < 16; ++l) {
        a0 = fmaf((float)u.q[l], x[l], a0);
        a1 = fmaf((float)u.q[l + 16], x[l + 16], a1);
    }
    float r = u.s0 * a0 + u.s1 * a1;
    if (u.has_off) {
#pragma unroll
        for (int l = 0; l < 32; ++l) sx += x[l];
        r = fmaf(u.off, sx, r);
    }
    return r;
}

// Runtime type dispatch helper: calls f(std::integral_constant<int, QT>{}) for
// a supported qt, returns false otherwise.
template <typename F>
__host__ inline bool sb_dispatch_qt(int qt, F&& f) {
    switch (qt) {
    case SB_Q5_1: f(std::integral_constant<int, SB_Q5_1>{}); return true;
    case SB_Q8_0: f(std::integral_constant<int, SB_Q8_0>{}); return true;
    case SB_Q4_K: f(std::integral_constant<int, SB_Q4_K>{}); return true;
    case SB_Q5_K: f(std::integral_constant<int, SB_Q5_K>{}); return true;
    case SB_Q6_K: f(std::integral_constant<int, SB_Q6_K>{}); return true;
    case SB_IQ3_XXS: f(std::integral_constant<int, SB_IQ3_XXS>{}); return true;
    case SB_IQ4_NL: f(std::integral_constant<int, SB_IQ4_NL>{}); return true;
    case SB_IQ3_S: f(std::integral_constant<int, SB_IQ3_S>{}); return true;
    case SB_IQ2_S: f(std::integral_constant<int, SB_IQ2_S>{}); return true;
    case SB_IQ4_XS: f(std::integral_constant<int, SB_IQ4_XS>{}); return true;
    case SB_Q2_0: f(std::integral_constant<int, SB_Q2_0>{}); return true;
    default: return false;
    }
}
