// Row movement for the expert-parallel bank: the (token, slot) pairs whose
// experts live on this GPU are gathered out of the all-gathered activations,
// pushed through the fused block as one "token" each, and their weighted
// outputs are summed back into token rows in a fixed order before the
// reduce-scatter. All three are plain copies / sums of a few hundred KB of
// fp32 rows: one thread per float4 of the output, so every load of a launch is
// in flight at once (the work is latency-bound, not bandwidth-bound).
#include <algorithm>

#include "sb_kernels.h"

#define SABAH_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr int kThreads = 256;   // 8 rows in flight per CTA

int sm_count() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms < 1) sms = 148;
    }
    return sms;
}
// one thread per float4 of the output, at most 8 CTAs per SM
int grid_elems(long long n4) { return (int)std::max(1LL, std::min((n4 + kThreads - 1) / kThreads, 8LL * sm_count())); }

// dst[i] = src[rows[i]]; a row index outside [0, n_src) gives a zero row, or,
// with err, a NaN row and SB_DERR_BAD_ID in *err
__global__ void k_gather_rows(const float4* src, int n_src, const int32_t* rows, int n, int k4, float4* dst, int* err) {
    const long long total = (long long)n * k4;
    for (long long q = blockIdx.x * (long long)kThreads + threadIdx.x; q < total; q += (long long)gridDim.x * kThreads) {
        const int i = (int)(q / k4), j = (int)(q % k4);
        const int r = __ldg(rows + i);
        if (r < 0 || r >= n_src) {
            const float f = err ? __int_as_float(0x7fc00000) : 0.f;
            if (err && j == 0) atomicExch(err, SB_DERR_BAD_ID);
            dst[q] = make_float4(f, f, f, f);
        } else {
            dst[q] = __ldg(src + (size_t)r * k4 + j);
        }
    }
}

// dst[t] = sum_{i in [off[t], off[t+1])} src[i], in increasing i (offsets
// clamped to [0, n_src]); the rows' loads are issued before the adds
__global__ void k_sum_rows(const float4* src, int n_src, const int32_t* off, int n_out, int k4, float4* dst) {
    const long long total = (long long)n_out * k4;
    for (long long q = blockIdx.x * (long long)kThreads + threadIdx.x; q < total; q += (long long)gridDim.x * kThreads) {
        const int t = (int)(q / k4), j = (int)(q % k4);
        const int i0 = max(__ldg(off + t), 0), i1 = min(__ldg(off + t + 1), n_src);
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        int i = i0;
        for (; i + 4 <= i1; i += 4) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = __ldg(src + (size_t)(i + u) * k4 + j);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                a.x += v[u].x;
                a.y += v[u].y;
                a.z += v[u].z;
                a.w += v[u].w;
            }
        }
        for (; i < i1; ++i) {
            const float4 v = __ldg(src + (size_t)i * k4 + j);
            a.x += v.x;
            a.y += v.y;
            a.z += v.z;
            a.w += v.w;
        }
        dst[q] = a;
    }
}

// dst[t] = init[t - i0] (t in [i0, i0 + n_init), else 0) + sum over
// i in [off[t], off[t+1]) of src[idx ? idx[i] : i], in increasing i: the pair
// sums of a layer with the residual folded in (an index outside [0, n_src)
// adds nothing). init may alias dst (same element, read before written).
__global__ void k_sum_rows_ex(const float4* src, int n_src, const int32_t* idx, const int32_t* off, int n_out, int k4,
                              float4* dst, const float4* init, int i0, int n_init) {
    const long long total = (long long)n_out * k4;
    for (long long q = blockIdx.x * (long long)kThreads + threadIdx.x; q < total; q += (long long)gridDim.x * kThreads) {
        const int t = (int)(q / k4), j = (int)(q % k4);
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        if (init && t >= i0 && t < i0 + n_init) a = init[(size_t)(t - i0) * k4 + j];
        const int b0 = __ldg(off + t), b1 = __ldg(off + t + 1);
        int i = b0;
        for (; i + 4 <= b1; i += 4) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int r = idx ? __ldg(idx + i + u) : i + u;
                v[u] = (r >= 0 && r < n_src) ? __ldg(src + (size_t)r * k4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                a.x += v[u].x;
                a.y += v[u].y;
                a.z += v[u].z;
                a.w += v[u].w;
            }
        }
        for (; i < b1; ++i) {
            const int r = idx ? __ldg(idx + i) : i;
            if (r < 0 || r >= n_src) continue;
            const float4 v = __ldg(src + (size_t)r * k4 + j);
            a.x += v.x;
            a.y += v.y;
            a.z += v.z;
            a.w += v.w;
        }
        dst[q] = a;
    }
}

// x += y
__global__ void k_add(float4* x, const float4* y, long long n4) {
    for (long long i = blockIdx.x * (long long)kThreads + threadIdx.x; i < n4; i += (long long)gridDim.x * kThreads) {
        const float4 a = x[i], b = __ldg(y + i);
        x[i] = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
    }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

int sb_gather_rows(const float* src, int n_src, const int32_t* rows, int n, int k, float* dst, int* err,
                   cudaStream_t st) {
    if (n <= 0) return 0;
    k_gather_rows<<<grid_elems((long long)n * (k / 4)), kThreads, 0, st>>>((const float4*)src, n_src, rows, n, k / 4,
                                                                         (float4*)dst, err);
    return sb_cuda_ok(cudaGetLastError(), "gather launch") ? 0 : -1;
}

SABAH_API int sabah_ep_gather_rows(const float* d_src, int n_src, const int32_t* d_rows, int n, int k,
                                   float* d_dst, void* stream) {
    if (n < 0 || n_src < 0 || k <= 0 || k % 4 || (n > 0 && (!d_src || !d_rows || !d_dst)) || !aligned16(d_src) ||
        !aligned16(d_dst)) {
        sb_set_error("invalid ep gather arguments (n %d, k %d)", n, k);
        return -1;
    }
    if (n == 0) return 0;
    const int tslot = sb_timing_begin("ep_gather_rows", (cudaStream_t)stream);
    k_gather_rows<<<grid_elems((long long)n * (k / 4)), kThreads, 0, (cudaStream_t)stream>>>(
        (const float4*)d_src, n_src, d_rows, n, k / 4, (float4*)d_dst, nullptr);
    sb_timing_end(tslot, (cudaStream_t)stream);
    return sb_cuda_ok(cudaGetLastError(), "ep gather launch") ? 0 : -1;
}

SABAH_API int sabah_ep_sum_rows(const float* d_src, int n_src, const int32_t* d_offsets, int n_out, int k,
                                float* d_dst, void* stream) {
    if (n_out < 0 || n_src < 0 || k <= 0 || k % 4 || (n_out > 0 && (!d_offsets || !d_dst)) ||
        (n_src > 0 && !d_src) || !aligned16(d_src) || !aligned16(d_dst)) {
        sb_set_error("invalid ep sum arguments (n_out %d, k %d)", n_out, k);
        return -1;
    }
    if (n_out == 0) return 0;
    const int tslot = sb_timing_begin("ep_sum_rows", (cudaStream_t)stream);
    k_sum_rows<<<grid_elems((long long)n_out * (k / 4)), kThreads, 0, (cudaStream_t)stream>>>(
        (const float4*)d_src, n_src, d_offsets, n_out, k / 4, (float4*)d_dst);
    sb_timing_end(tslot, (cudaStream_t)stream);
    return sb_cuda_ok(cudaGetLastError(), "ep sum launch") ? 0 : -1;
}

SABAH_API int sabah_ep_add(float* d_x, const float* d_y, long long n, void* stream) {
    if (n < 0 || n % 4 || (n > 0 && (!d_x || !d_y)) || !aligned16(d_x) || !aligned16(d_y)) {
        sb_set_error("invalid ep add arguments (n %lld)", n);
        return -1;
    }
    if (n == 0) return 0;
    const int tslot = sb_timing_begin("ep_add", (cudaStream_t)stream);
    k_add<<<grid_elems(n / 4), kThreads, 0, (cudaStream_t)stream>>>((float4*)d_x, (const float4*)d_y, n / 4);
    sb_timing_end(tslot, (cudaStream_t)stream);
    return sb_cuda_ok(cudaGetLastError(), "ep add launch") ? 0 : -1;
}

SABAH_API int sabah_ep_sum_rows_ex(const float* d_src, int n_src, const int32_t* d_idx, const int32_t* d_offsets,
                                   int n_out, int k, float* d_dst, const float* d_init, int init_row0, int n_init,
                                   void* stream) {
    if (n_out < 0 || n_src < 0 || k <= 0 || k % 4 || n_init < 0 || (n_out > 0 && (!d_offsets || !d_dst)) ||
        (n_src > 0 && !d_src) || (n_init > 0 && !d_init) || !aligned16(d_src) || !aligned16(d_dst) ||
        !aligned16(d_init)) {
        sb_set_error("invalid ep sum_ex arguments (n_out %d, k %d, n_init %d)", n_out, k, n_init);
        return -1;
    }
    if (n_out == 0) return 0;
    const int tslot = sb_timing_begin("ep_sum_rows", (cudaStream_t)stream);
    k_sum_rows_ex<<<grid_elems((long long)n_out * (k / 4)), kThreads, 0, (cudaStream_t)stream>>>(
        (const float4*)d_src, n_src, d_idx, d_offsets, n_out, k / 4, (float4*)d_dst,
        n_init > 0 ? (const float4*)d_init : nullptr, init_row0, n_init);
    sb_timing_end(tslot, (cudaStream_t)stream);
    return sb_cuda_ok(cudaGetLastError(), "ep sum_ex launch") ? 0 : -1;
}
