// Synthetic expert banks, encoded on the device.
//
// Weights are N(0, sigma) drawn from a counter-based generator (splitmix64 of
// (seed, element index) -> Box-Muller), so any sub-range of a bank can be
// regenerated independently and the same seed always gives the same bytes.
// The encoders are this project's own (ggml's Q4_K/Q6_K/IQ3_S quantizers are
// not part of it); they produce valid blocks of each format from the block
// layouts. Q8_0 follows ggml's reference rule (d = amax/127, q = roundf(v/d)).
// Parity never depends on encoder quality: the bytes a kernel reads are the
// bytes the oracle reads.
#include <cmath>
#include <cstdio>
#include <vector>

#include "sb_kernels.h"
#include "sb_quant.cuh"

#define SABAH_API extern "C" __attribute__((visibility("default")))

namespace {

__device__ inline uint64_t mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ inline float normal_at(uint64_t seed, uint64_t n, float sigma) {
    const uint64_t h = mix(seed * 0xD1B54A32D192ED03ull ^ mix(n));
    const float u1 = ((float)(uint32_t)(h >> 40) + 1.0f) * (1.0f / 16777217.0f);   // (0, 1]
    const float u2 = (float)(uint32_t)(h & 0xFFFFFFu) * (1.0f / 16777216.0f);
    return sigma * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__device__ inline uint16_t f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ inline float f16_round(float v) { return __half2float(__float2half_rn(v)); }
__device__ inline void put16(uint8_t* p, uint16_t v) {
    p[0] = (uint8_t)(v & 255);
    p[1] = (uint8_t)(v >> 8);
}

// nearest IQ3_S grid entry for each of the 4096 level 4-tuples (3 bits each,
// level L stands for the odd value 2L + 1)
__global__ void k_iq3s_nearest(uint16_t* out) {
    const int code = blockIdx.x * blockDim.x + threadIdx.x;
    if (code >= 4096) return;
    int best = 0, best_d = 1 << 30;
    for (int g = 0; g < 512; ++g) {
        const uint32_t w = sb_iq3s_grid[g];
        int dist = 0;
        for (int i = 0; i < 4; ++i) {
            const int want = 2 * ((code >> (3 * i)) & 7) + 1;
            const int have = (int)((w >> (8 * i)) & 255);
            dist += (want - have) * (want - have);
        }
        if (dist < best_d) {
            best_d = dist;
            best = g;
        }
    }
    out[code] = (uint16_t)best;
}

// One thread encodes one block. Element n of the tensor is (row0 + row) * k +
// column, so rows [row0, row0 + n_rows) of a larger tensor can be made alone.
template <int QT>
__global__ void k_synth(uint8_t* dst, long long row0, long long n_rows, int k, uint64_t seed, float sigma,
                        const uint16_t* nearest) {
    const int be = sb_block_elems(QT), bb = sb_block_bytes(QT);
    const int bpr = k / be;
    const long long nblk = n_rows * bpr;
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nblk; b += (long long)gridDim.x * blockDim.x) {
        const long long row = b / bpr;
        const int col0 = (int)(b % bpr) * be;
        const uint64_t n0 = (uint64_t)(row0 + row) * (uint64_t)k + (uint64_t)col0;
        uint8_t* o = dst + (size_t)b * bb;
        auto v = [&](int i) { return normal_at(seed, n0 + (uint64_t)i, sigma); };
        if constexpr (QT == SB_Q8_0) {
            float amax = 0.f;
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v(i)));
            const float d = amax / 127.f, id = d != 0.f ? 1.f / d : 0.f;
            put16(o, f16_bits(d));
            for (int i = 0; i < 32; ++i) o[2 + i] = (uint8_t)(int8_t)roundf(v(i) * id);
        } else if constexpr (QT == SB_IQ3_S) {
            float sub_s[8], smax = 0.f;
            for (int j = 0; j < 8; ++j) {
                float amax = 0.f;
                for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v(32 * j + i)));
                sub_s[j] = amax / 15.f;
                smax = fmaxf(smax, sub_s[j]);
            }
            const float d = f16_round(smax / 31.f);
            put16(o, f16_bits(d));
            for (int i = 2; i < 110; ++i) o[i] = 0;
            for (int j = 0; j < 8; ++j) {
                int sc = d > 0.f ? (int)rintf((sub_s[j] / d - 1.f) * 0.5f) : 0;
                sc = min(max(sc, 0), 15);
                o[106 + j / 2] |= (uint8_t)(sc << (4 * (j & 1)));
                const float db = d * (float)(1 + 2 * sc);
                const float idb = db > 0.f ? 1.f / db : 0.f;
                for (int g = 0; g < 8; ++g) {            // 8 groups of 4 values
                    int code = 0;
                    for (int i = 0; i < 4; ++i) {
                        const float x = v(32 * j + 4 * g + i);
                        int L = (int)rintf((fabsf(x) * idb - 1.f) * 0.5f);
                        L = min(max(L, 0), 7);
                        code |= L << (3 * i);
                        if (x < 0.f) o[74 + 4 * j + g / 2] |= (uint8_t)(1 << (4 * (g & 1) + i));
                    }
                    const int gi = nearest[code];
                    o[2 + 8 * j + g] = (uint8_t)(gi & 255);
                    o[66 + j] |= (uint8_t)((gi >> 8) << g);
                }
            }
        } else if constexpr (QT == SB_Q4_K) {
            float scl[8], mins[8], smax = 0.f, mmax = 0.f;
            for (int j = 0; j < 8; ++j) {
                float lo = 0.f, hi = 0.f;
                for (int i = 0; i < 32; ++i) {
                    const float x = v(32 * j + i);
                    lo = fminf(lo, x);
                    hi = fmaxf(hi, x);
                }
                scl[j] = (hi - lo) / 15.f;
                mins[j] = -lo;
                smax = fmaxf(smax, scl[j]);
                mmax = fmaxf(mmax, mins[j]);
            }
            const float d = f16_round(smax / 63.f), dmin = f16_round(mmax / 63.f);
            put16(o, f16_bits(d));
            put16(o + 2, f16_bits(dmin));
            int s6[8], m6[8];
            for (int j = 0; j < 8; ++j) {
                s6[j] = d > 0.f ? min(63, max(0, (int)rintf(scl[j] / d))) : 0;
                m6[j] = dmin > 0.f ? min(63, max(0, (int)rintf(mins[j] / dmin))) : 0;
            }
            for (int j = 0; j < 4; ++j) {
                o[4 + j] = (uint8_t)((s6[j] & 63) | ((s6[j + 4] >> 4) << 6));
                o[8 + j] = (uint8_t)((m6[j] & 63) | ((m6[j + 4] >> 4) << 6));
                o[12 + j] = (uint8_t)((s6[j + 4] & 15) | ((m6[j + 4] & 15) << 4));
            }
            for (int i = 16; i < 144; ++i) o[i] = 0;
            for (int j = 0; j < 8; ++j) {
                const float ds = d * (float)s6[j], dm = dmin * (float)m6[j];
                const float ids = ds > 0.f ? 1.f / ds : 0.f;
                for (int l = 0; l < 32; ++l) {
                    int q = (int)rintf((v(32 * j + l) + dm) * ids);
                    q = min(max(q, 0), 15);
                    o[16 + 32 * (j >> 1) + l] |= (uint8_t)(q << (4 * (j & 1)));
                }
            }
        } else if constexpr (QT == SB_Q6_K) {
            float scl[16], smax = 0.f;
            for (int i = 0; i < 16; ++i) {
                float amax = 0.f;
                for (int l = 0; l < 16; ++l) amax = fmaxf(amax, fabsf(v(16 * i + l)));
                scl[i] = amax / 31.f;
                smax = fmaxf(smax, scl[i]);
            }
            const float d = f16_round(smax / 127.f);
            put16(o + 208, f16_bits(d));
            for (int i = 0; i < 192; ++i) o[i] = 0;
            for (int i = 0; i < 16; ++i) {
                const int sc = d > 0.f ? min(127, max(1, (int)rintf(scl[i] / d))) : 0;
                o[192 + i] = (uint8_t)(int8_t)sc;
                const float ds = d * (float)sc, ids = ds > 0.f ? 1.f / ds : 0.f;
                for (int l = 0; l < 16; ++l) {
                    const int e = 16 * i + l;
                    int q = (int)rintf(v(e) * ids);
                    q = min(max(q, -32), 31) + 32;
                    const int h = e >> 7, ep = e & 127, p = ep >> 5, ll = ep & 31;
                    o[64 * h + 32 * (p & 1) + ll] |= (uint8_t)((q & 15) << (4 * (p >> 1)));
                    o[128 + 32 * h + ll] |= (uint8_t)((q >> 4) << (2 * p));
                }
            }
        }
    }
}

uint16_t* g_nearest = nullptr;

}  // namespace

// Fill d_dst with rows [row0, row0 + n_rows) of a tensor of rows of k elements
// of type qt (dense rows), weights N(0, sigma) from `seed`. Supported: Q8_0,
// Q4_K, Q6_K, IQ3_S. Asynchronous on `stream` (NULL: the legacy default stream).
SABAH_API int sabah_synth_rows_at(void* d_dst, int qt, long long row0, long long n_rows, int k,
                                  unsigned long long seed, float sigma, void* stream) {
    if (!d_dst || n_rows < 0 || row0 < 0 || k <= 0 || !sb_row_bytes_of(qt, k)) {
        sb_set_error("invalid synth geometry (type %d, k %d)", qt, k);
        return -1;
    }
    cudaStream_t st = (cudaStream_t)stream;
    if (qt == SB_IQ3_S && !g_nearest) {
        if (!sb_cuda_ok(cudaMalloc(&g_nearest, 4096 * sizeof(uint16_t)), "synth table")) return -1;
        k_iq3s_nearest<<<16, 256, 0, st>>>(g_nearest);
    }
    const long long nblk = n_rows * (k / sb_block_elems(qt));
    const int grid = (int)std::min<long long>((nblk + 255) / 256, 148LL * 64);
    uint8_t* d = (uint8_t*)d_dst;
    switch (qt) {
    case SB_Q8_0: k_synth<SB_Q8_0><<<grid, 256, 0, st>>>(d, row0, n_rows, k, seed, sigma, g_nearest); break;
    case SB_Q4_K: k_synth<SB_Q4_K><<<grid, 256, 0, st>>>(d, row0, n_rows, k, seed, sigma, g_nearest); break;
    case SB_Q6_K: k_synth<SB_Q6_K><<<grid, 256, 0, st>>>(d, row0, n_rows, k, seed, sigma, g_nearest); break;
    case SB_IQ3_S: k_synth<SB_IQ3_S><<<grid, 256, 0, st>>>(d, row0, n_rows, k, seed, sigma, g_nearest); break;
    default:
        sb_set_error("synth: quant type %d has no encoder", qt);
        return -1;
    }
    return sb_cuda_ok(cudaGetLastError(), "synth launch") ? 0 : -1;
}

SABAH_API int sabah_synth_rows(void* d_dst, int qt, long long n_rows, int k, unsigned long long seed, float sigma,
                               void* stream) {
    return sabah_synth_rows_at(d_dst, qt, 0, n_rows, k, seed, sigma, stream);
}
