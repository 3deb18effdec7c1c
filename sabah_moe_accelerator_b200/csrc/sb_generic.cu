// Generic kernels for every supported expert quant type: the MUL_MAT_ID
// matvec, the bit-exact dequantizer and the fused routed block. One warp owns
// an output row; its lanes stride over the row's 32-element sub-blocks, decode
// them in registers (sb_quant.cuh) and reduce with shuffles. Types with a
// tensor-core fast path (sb_mmid_iq3s.cu) only come here for shapes that path
// does not cover.
#include <cmath>

#include "sb_kernels.h"
#include "sb_quant.cuh"

namespace {

constexpr int kWarps = 8;          // 256 threads per CTA
constexpr int kRowsPerCta = 32;    // each warp takes every 8th row of the tile

__device__ inline float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Expert base for (token t, slot i), or nullptr when the router id is outside
// [0, n_experts) (recorded in *err).
__device__ inline const uint8_t* expert_of(const sb_experts& e, int t, int i, int n_ids, int* err) {
    if (e.ptrs) return (const uint8_t*)e.ptrs[(size_t)t * n_ids + i];
    int id = *(const int32_t*)((const uint8_t*)e.ids + (size_t)t * e.ids_token_stride + (size_t)i * e.ids_id_stride);
#if SABAH_SENTINEL == 1
    // test-only build: slot 0 runs the neighbouring expert
    if (i == 0 && id >= 0 && id < e.n_experts) id = (id + 1) % e.n_experts;
#endif
    if (id < 0 || id >= e.n_experts) {
        if (err) atomicExch(err, SB_DERR_BAD_ID);
        return nullptr;
    }
    return e.base + (size_t)id * e.expert_stride;
}

__device__ inline void load_x32(const float* x, float (&xs)[32]) {
    const float4* p = reinterpret_cast<const float4*>(x);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 v = __ldg(p + q);
        xs[4 * q] = v.x;
        xs[4 * q + 1] = v.y;
        xs[4 * q + 2] = v.z;
        xs[4 * q + 3] = v.w;
    }
}

template <int QT>
__device__ inline float row_dot(const uint8_t* row, const float* x, int nsub, int lane) {
    float acc = 0.f;
    for (int s = lane; s < nsub; s += 32) {
        float xs[32];
        load_x32(x + 32 * s, xs);
        acc += sb_dot32<QT>(row, s, xs);
    }
    return warp_sum(acc);
}

// grid (ceil(rows / 32), n_ids, n_tokens), 256 threads
template <int QT>
__global__ void __launch_bounds__(256) k_mmid_generic(sb_mmid_args a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i = blockIdx.y, t = blockIdx.z;
    const uint8_t* w = expert_of(a.ex, t, i, a.n_ids, a.err);
#if SABAH_SENTINEL == 2
    const int xr = a.x_rows > 1 ? (i + 1) % a.x_rows : 0;   // test-only: wrong input row
#else
    const int xr = i % a.x_rows;
#endif
#if SABAH_SENTINEL == 3
    const int xt = (t + 1) % a.n_tokens;                      // test-only: wrong token
#else
    const int xt = t;
#endif
    const float* x = (const float*)((const uint8_t*)a.x + (size_t)xr * a.x_id_stride + (size_t)xt * a.x_token_stride);
    float* dst = (float*)((uint8_t*)a.dst + (size_t)t * a.dst_token_stride + (size_t)i * a.dst_id_stride);
    const int r_end = min(a.rows, (int)(blockIdx.x + 1) * kRowsPerCta);
    const int nsub = a.k / 32;
    for (int r = blockIdx.x * kRowsPerCta + warp; r < r_end; r += kWarps) {
        float v = w ? row_dot<QT>(w + (size_t)r * a.row_stride, x, nsub, lane) : __int_as_float(0x7fc00000);
        if (lane == 0) dst[r] = v;
    }
}

// one thread per 32-element sub-block
template <int QT>
__global__ void k_dequant(const uint8_t* src, float* dst, int n_rows, int row_elems) {
    const int nsub = row_elems / 32;
    const size_t rb = sb_row_bytes_of(QT, row_elems);
    const size_t total = (size_t)n_rows * nsub;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t r = idx / nsub;
        const int s = (int)(idx % nsub);
        float y[32];
        sb_dequant32<QT>(src + r * rb, s, y);
        float4* o = reinterpret_cast<float4*>(dst + r * row_elems + 32 * s);
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
    }
}

__device__ inline float silu_mul(float g, float u) { return g / (1.f + __expf(-g)) * u; }

// h[t][e][j] = silu(<Wg[e][j], x_t>) * <Wu[e][j], x_t>
// grid (ceil(ff / 32), n_used, n_tokens), 256 threads
template <int QG, int QU>
__global__ void __launch_bounds__(256) k_gate_up_generic(sb_block_args a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.y, t = blockIdx.z;
    const uint8_t* wg = expert_of(a.gate, t, e, a.n_used, a.err);
    const uint8_t* wu = expert_of(a.up, t, e, a.n_used, a.err);
    const float* x = a.x + (size_t)t * a.d_model;
    float* h = a.h + ((size_t)t * a.n_used + e) * a.ff;
    const size_t rbg = sb_row_bytes_of(QG, a.d_model), rbu = sb_row_bytes_of(QU, a.d_model);
    const int nsub = a.d_model / 32;
    const int r_end = min(a.ff, (int)(blockIdx.x + 1) * kRowsPerCta);
    for (int j = blockIdx.x * kRowsPerCta + warp; j < r_end; j += kWarps) {
        float v = __int_as_float(0x7fc00000);
        if (wg && wu) {
            const float g = row_dot<QG>(wg + (size_t)j * rbg, x, nsub, lane);
            const float u = row_dot<QU>(wu + (size_t)j * rbu, x, nsub, lane);
            v = silu_mul(g, u);
        }
        if (lane == 0) h[j] = v;
    }
}

// out[t][i] (+)= sum_e w[t][e] * <Wd[e][i], h[t][e]>, experts summed in slot
// order by one warp (deterministic, no atomics).
// grid (ceil(d_model / 32), 1, n_tokens), 256 threads
template <int QD>
__global__ void __launch_bounds__(256) k_down_generic(sb_block_args a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.z;
    const size_t rbd = sb_row_bytes_of(QD, a.ff);
    const int nsub = a.ff / 32;
    const int r_end = min(a.d_model, (int)(blockIdx.x + 1) * kRowsPerCta);
    for (int i = blockIdx.x * kRowsPerCta + warp; i < r_end; i += kWarps) {
        float total = 0.f;
        for (int e = 0; e < a.n_used; ++e) {
            const uint8_t* wd = expert_of(a.down, t, e, a.n_used, a.err);
            const float* h = a.h + ((size_t)t * a.n_used + e) * a.ff;
            const float v = wd ? row_dot<QD>(wd + (size_t)i * rbd, h, nsub, lane) : __int_as_float(0x7fc00000);
            total = fmaf(a.w[(size_t)t * a.n_used + e], v, total);
        }
        if (lane == 0) {
            float* o = a.out + (size_t)t * a.d_model + i;
            *o = a.accumulate ? *o + total : total;
        }
    }
}

// gate and up of different types: the gate pass leaves g in h, the up pass
// turns it into silu(g) * u in place.
template <int QT, bool kSwiglu>
__global__ void __launch_bounds__(256) k_half_generic(sb_block_args a, const sb_experts ex) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e = blockIdx.y, t = blockIdx.z;
    const uint8_t* w = expert_of(ex, t, e, a.n_used, a.err);
    const float* x = a.x + (size_t)t * a.d_model;
    float* h = a.h + ((size_t)t * a.n_used + e) * a.ff;
    const size_t rb = sb_row_bytes_of(QT, a.d_model);
    const int nsub = a.d_model / 32;
    const int r_end = min(a.ff, (int)(blockIdx.x + 1) * kRowsPerCta);
    for (int j = blockIdx.x * kRowsPerCta + warp; j < r_end; j += kWarps) {
        float v = w ? row_dot<QT>(w + (size_t)j * rb, x, nsub, lane) : __int_as_float(0x7fc00000);
        if (lane == 0) h[j] = kSwiglu ? silu_mul(h[j], v) : v;
    }
}

}  // namespace

bool sb_qt_supported(int qt) { return sb_block_elems(qt) != 0; }

int sb_launch_mmid(const sb_mmid_args& a, cudaStream_t st) {
    const int taken = sb_try_mmid_iq3s(a, st);
    if (taken != 0) return taken > 0 ? 0 : -1;
    const int q8 = sb_try_mmid_q8_0(a, st);
    if (q8 != 0) return q8 > 0 ? 0 : -1;
    dim3 grid((a.rows + kRowsPerCta - 1) / kRowsPerCta, a.n_ids, a.n_tokens);
    auto l = [&](auto tag) { k_mmid_generic<decltype(tag)::value><<<grid, 256, 0, st>>>(a); };
    const int tslot = sb_timing_begin("mmid_generic", st);
    const bool ok = sb_dispatch_qt(a.qt, l);
    sb_timing_end(tslot, st);
    if (!ok) {
        sb_set_error("unsupported quant type %d", a.qt);
        return -1;
    }
    return sb_cuda_ok(cudaGetLastError(), "MUL_MAT_ID launch") ? 0 : -1;
}

int sb_launch_dequant(const void* src, float* dst, int qt, int n_rows, int row_elems, cudaStream_t st) {
    const long long subs = (long long)n_rows * (row_elems / 32);
    const int grid = (int)std::min<long long>((subs + 255) / 256, 148LL * 16);
    const int g = grid > 0 ? grid : 1;
    auto l = [&](auto tag) {
        k_dequant<decltype(tag)::value><<<g, 256, 0, st>>>((const uint8_t*)src, dst, n_rows, row_elems);
    };
    if (!sb_dispatch_qt(qt, l)) {
        sb_set_error("unsupported quant type %d", qt);
        return -1;
    }
    return sb_cuda_ok(cudaGetLastError(), "dequant launch") ? 0 : -1;
}

int sb_launch_block(const sb_block_args& a, cudaStream_t st) {
    const int taken = sb_try_block_iq3s(a, st);
    if (taken != 0) return taken > 0 ? 0 : -1;
    const int small = sb_try_block_small(a, st);
    if (small != 0) return small > 0 ? 0 : -1;
    const int q8 = sb_try_block_q8_0(a, st);
    if (q8 != 0) return q8 > 0 ? 0 : -1;
    dim3 g1((a.ff + kRowsPerCta - 1) / kRowsPerCta, a.n_used, a.n_tokens);
    bool ok;
    const int t1 = sb_timing_begin("gate_up_generic", st);
    if (a.qt_gate == a.qt_up) {
        auto l = [&](auto tag) {
            constexpr int QT = decltype(tag)::value;
            k_gate_up_generic<QT, QT><<<g1, 256, 0, st>>>(a);
        };
        ok = sb_dispatch_qt(a.qt_gate, l);
    } else {
        auto lg = [&](auto tag) { k_half_generic<decltype(tag)::value, false><<<g1, 256, 0, st>>>(a, a.gate); };
        auto lu = [&](auto tag) { k_half_generic<decltype(tag)::value, true><<<g1, 256, 0, st>>>(a, a.up); };
        ok = sb_dispatch_qt(a.qt_gate, lg) && sb_dispatch_qt(a.qt_up, lu);
    }
    sb_timing_end(t1, st);
    if (!ok) {
        sb_set_error("unsupported gate/up quant type %d/%d", a.qt_gate, a.qt_up);
        return -1;
    }
    dim3 g2((a.d_model + kRowsPerCta - 1) / kRowsPerCta, 1, a.n_tokens);
    auto ld = [&](auto tag) { k_down_generic<decltype(tag)::value><<<g2, 256, 0, st>>>(a); };
    const int t2 = sb_timing_begin("down_generic", st);
    const bool okd = sb_dispatch_qt(a.qt_down, ld);
    sb_timing_end(t2, st);
    if (!okd) {
        sb_set_error("unsupported down quant type %d", a.qt_down);
        return -1;
    }
    return sb_cuda_ok(cudaGetLastError(), "moe block launch") ? 0 : -1;
}
