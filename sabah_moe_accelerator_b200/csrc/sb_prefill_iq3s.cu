// Grouped IQ3_S MUL_MAT_ID for prefill on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in TMEM).
//
// With many tokens per call, MUL_MAT_ID is a grouped GEMM: expert e multiplies
// its matrix W_e [rows][k] by the x rows of the n_e (token, slot) pairs routed
// to it. The (token, slot) pairs are grouped by expert on the device (count,
// scan, scatter). Experts with more than 8 pairs go to the tcgen05 kernel
// below, which walks tasks (expert, 128-row tile, up to 128 pairs); experts
// with 1-8 pairs go to a register-decode kernel (mma.sync, further down),
// because a 128-wide MMA tile would be mostly padding for them. Both run in
// one stream, back to back. In the tcgen05 kernel:
//
// * the tile's raw IQ3_S rows (128 x row bytes, contiguous in the bank) land in
//   shared memory with one cp.async.bulk: every weight byte is read from HBM
//   once per task;
// * per 32-wide K slice (one IQ3_S sub-block), 256 threads dequantise A (128 x
//   32) and convert B (the pairs' x, up to 256 x 32) into the K-major
//   "interleaved" core-matrix layout (8 rows x 16 bytes per core matrix), double
//   buffered;
// * one thread issues the slice's MMAs (M = 128, N = pairs rounded to 16, K = 16
//   each) into one TMEM accumulator and commits them to the stage's mbarrier;
// * precision: A and B are each split into fp16 hi + lo parts and the MMAs
//   compute hi*hi + hi*lo + lo*hi (fp32 accumulate), so products are good to
//   ~2^-21 relative, fp32-grade like the reference's fp32 FMA kernels. Each
//   weight row and each x row is scaled by a power of two into fp16's range
//   first (undone exactly in the epilogue);
// * epilogue: tcgen05.ld (32 lanes x 32-bit) of the accumulator, one output
//   row per TMEM lane, written straight to dst[token][slot][row].
//
// Every wait is bounded; on timeout the CTA records SB_DERR_TIMEOUT, stops
// issuing work, and still frees its TMEM.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "sb_kernels.h"
#include "sb_quant.cuh"

namespace {

// Warp roles: warps 0-7 (the producers) each slice dequantise A (thread t:
// row t % 128, half the sub-block's grid entries) from the task's raw tile in
// shared memory and convert B (the pairs' x, 8-wide chunks); warp 8 owns TMEM
// and issues the MMAs (lane 0). Warps 0-7 run the epilogue. Stages move
// between them through full / empty mbarriers.
constexpr int kProducers = 256;                   // warps 0-7
constexpr int kThreads = kProducers + 32;         // + the MMA warp
constexpr int kM = 128;                           // rows per task (MMA M)
constexpr int kMaxN = 128;                        // pairs per task (MMA N, TMEM columns)
constexpr int kKs = 32;                           // K slice: one IQ3_S sub-block
constexpr int kStages = 3;
constexpr int kRawBytes = kM * 880;               // raw tile, k <= 2048
constexpr int kAHalf = kM * kKs * 2;              // 8 KB: one fp16 A operand of a slice
constexpr int kBHalf = kMaxN * kKs * 2;           // 16 KB: one fp16 B operand of a slice
constexpr int kStageBytes = 2 * kAHalf + 2 * kBHalf;
constexpr int kGridReplicas = 8;
constexpr long long kSpinLimit = 1ll << 26;
constexpr int kGMaxPairs = 8;                     // pairs per register-decode task (the MMA's 8 columns)

struct Smem {
    static constexpr int raw = 0;                                             // the task's weight tile
    static constexpr int grid = raw + kRawBytes;                              // [512][kGridReplicas] u32
    static constexpr int stage = (grid + 512 * kGridReplicas * 4 + 1023) & ~1023;   // [kStages] {A_hi, A_lo, B_hi, B_lo}
    static constexpr int row_exp = stage + kStages * kStageBytes;             // [kM] int
    static constexpr int pair_exp = row_exp + kM * 4;                         // [kMaxN] int
    static constexpr int pair_dst = pair_exp + kMaxN * 4;                     // [kMaxN] float*
    static constexpr int bars = pair_dst + kMaxN * 8;                         // full[kStages], empty[kStages], tfull, tempty, done, raw
    static constexpr int tmem_base = bars + (2 * kStages + 4) * 8;
    static constexpr int flags = tmem_base + 8;                               // abort
    static constexpr int total = flags + 8;
};
static_assert(Smem::total <= 227 * 1024, "shared memory budget");

struct Task {
    int expert, mt, n0, n;   // expert, 128-row tile, first pair (in the grouped order), pairs
};

struct PairInfo {
    long long x_off;    // byte offset of the pair's x row
    long long dst_off;  // byte offset of the pair's dst row
    int exp;            // x scale: the row is multiplied by 2^exp before the fp16 split
    int xrow;           // the x row: t * x_rows + i % x_rows
};

struct GemmParams {
    const uint8_t* base;         // bank
    size_t expert_stride;        // bytes
    int rb, k, rows;
    const uint8_t* x;            // fp32 rows
    uint8_t* dst;                // fp32 rows
    const Task* tasks;
    const int* n_tasks;
    const PairInfo* pairs;       // grouped order
    int* err;
};

__device__ inline uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ inline bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait. False when the CTA is aborting or when this wait gives up (it
// then sets the abort flag and the error word).
__device__ inline bool mbar_wait(uint32_t bar, uint32_t parity, int* err, volatile int* abort_flag) {
    for (long long i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 63 && *abort_flag) return false;
    }
    *abort_flag = 1;
    if (err) atomicExch(err, SB_DERR_TIMEOUT);
    return false;
}
__device__ inline void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ inline void producers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kProducers) : "memory"); }
// bring a contiguous byte range (16-byte aligned, size a multiple of 16) into L2
__device__ inline void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}


// Shared-memory matrix descriptor, K-major, no swizzle: core matrices of 8
// rows x 16 bytes (rows 16 bytes apart); lbo = bytes between the two K halves
// of an MMA (adjacent core matrices along K), sbo = bytes between adjacent
// 8-row groups. Version 1 (tcgen05).
__device__ inline uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

// Instruction descriptor, kind::f16: D f32, A and B f16, both K-major, M x N.
__device__ inline uint32_t instr_desc(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ inline void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ inline void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane
__device__ inline void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Offset of 16-byte chunk (row, k-chunk c) in an operand of `rows` rows laid
// out K-major interleaved: chunk-major over K, then 8-row groups.
__device__ inline uint32_t chunk_off(int row, int c, int rows) {
    return (uint32_t)(((c * (rows >> 3) + (row >> 3)) << 7) + ((row & 7) << 4));
}

// hi/lo fp16 split of 8 floats into two 16-byte chunks. hi keeps the top 11
// significant bits (mantissa truncated, so it is exact in fp16 for values in
// fp16's normal range, which the power-of-two row and pair scales provide);
// lo = v - hi is exact in fp32 and rounded to fp16. One paired conversion per
// two values for each part.
__device__ inline void split8(const float (&v)[8], uint4& hi, uint4& lo) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float a = v[2 * i], b = v[2 * i + 1];
        const float ah = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
        const float bh = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
        const __half2 hh = __floats2half2_rn(ah, bh), ll = __floats2half2_rn(a - ah, b - bh);
        h[i] = *(const uint32_t*)&hh;
        l[i] = *(const uint32_t*)&ll;
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

__device__ inline uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ inline float f16_bits(unsigned v) { return __half2float(__ushort_as_half((unsigned short)v)); }

__global__ void __launch_bounds__(kThreads, 1) k_prefill_iq3s(const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    uint64_t* bars = (uint64_t*)(smem + Smem::bars);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStages);
    const uint32_t tfull = smem_u32(bars + 2 * kStages), tempty = tfull + 8, done = tfull + 16, rawbar = tfull + 24;
    volatile int* abort_flag = (volatile int*)(smem + Smem::flags);
    int* row_exp = (int*)(smem + Smem::row_exp);
    int* pair_exp = (int*)(smem + Smem::pair_exp);
    float** pair_dst = (float**)(smem + Smem::pair_dst);
    uint32_t* gtab = (uint32_t*)(smem + Smem::grid);
    // the register-decode kernel launched after this one reads nothing this
    // kernel writes: its CTAs may take the SMs this kernel's CTAs leave
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (tid == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * s), "r"(kProducers / 32));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(empty0 + 8 * s));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tfull));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tempty), "r"(kProducers / 32));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(done));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(rawbar));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int e = tid; e < 512; e += kThreads) {
        const uint32_t w = sb_iq3s_grid[e];
#pragma unroll
        for (int r = 0; r < kGridReplicas; ++r) gtab[e * kGridReplicas + r] = w;
    }
    if (warp == kProducers / 32) {   // TMEM: kMaxN fp32 columns x 128 lanes, one accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(smem + Smem::tmem_base)),
                     "r"(kMaxN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *(volatile uint32_t*)(smem + Smem::tmem_base);
    const int n_tasks = *p.n_tasks;
    const int nk = p.k / kKs;   // K slices per task
    const uint32_t stage0 = smem_u32(smem + Smem::stage);
    const uint32_t tile_bytes = (uint32_t)(kM * p.rb);
    // raw tile of task ti into shared memory (one thread)
    auto issue_raw = [&](int ti) {
        const Task tn = p.tasks[ti];
        const uint8_t* src = p.base + (size_t)tn.expert * p.expert_stride + (size_t)tn.mt * kM * p.rb;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // earlier generic reads of the tile
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(rawbar), "r"(tile_bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_u32(smem + Smem::raw)),
                     "l"(src), "r"(tile_bytes), "r"(rawbar)
                     : "memory");
    };
    int raw_issued = 0, raw_waited = 0;   // thread 0's count of tile copies
    if (tid == 0 && (int)blockIdx.x < n_tasks) {
        issue_raw(blockIdx.x);
        ++raw_issued;
    }

    if (warp == kProducers / 32) {
        // ---------------------------------------------------------- MMA warp
        if (lane == 0) {
            int g = 0, i = 0;
            for (int ti = blockIdx.x; ti < n_tasks; ti += gridDim.x, ++i) {
                const Task t = p.tasks[ti];
                const uint32_t idesc = instr_desc(kM, (t.n + 15) & ~15);
                // the previous task's accumulator has been read out
                if (i > 0 && !mbar_wait(tempty, (i - 1) & 1, p.err, abort_flag)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                bool ok = true;
                for (int kt = 0; kt < nk; ++kt, ++g) {
                    const int s = g % kStages;
                    if (!mbar_wait(full0 + 8 * s, (g / kStages) & 1, p.err, abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t sa = stage0 + s * kStageBytes;
                    const uint32_t a_hi = sa, a_lo = sa + kAHalf, b_hi = sa + 2 * kAHalf, b_lo = b_hi + kBHalf;
                    constexpr uint32_t a_lbo = (kM / 8) * 128, b_lbo = (kMaxN / 8) * 128;   // bytes between K halves
#pragma unroll
                    for (int ks = 0; ks < kKs / 16; ++ks) {
                        const uint32_t ao = ks * 2 * a_lbo, bo = ks * 2 * b_lbo;
                        const uint32_t acc0 = (kt > 0 || ks > 0) ? 1u : 0u;
                        mma_f16(tmem, smem_desc(a_hi + ao, a_lbo, 128), smem_desc(b_hi + bo, b_lbo, 128), idesc, acc0);
                        mma_f16(tmem, smem_desc(a_hi + ao, a_lbo, 128), smem_desc(b_lo + bo, b_lbo, 128), idesc, 1u);
                        mma_f16(tmem, smem_desc(a_lo + ao, a_lbo, 128), smem_desc(b_hi + bo, b_lbo, 128), idesc, 1u);
                    }
                    mma_commit(empty0 + 8 * s);   // the stage is free once these MMAs are done
                }
                if (!ok) break;
                mma_commit(tfull);                // the accumulator is complete
            }
            // never leave with MMAs in flight (TMEM is freed below)
            mma_commit(done);
            for (long long it = 0; it < kSpinLimit && !mbar_try_wait(done, 0); ++it) {
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------- producers (warps 0-7)
        // every producer thread does both jobs each slice:
        //   A: rows r1 = 16 warp + (lane & 7) and r1 + 8, quarter aq = lane / 8 of the
        //      slice's sub-block (entries 2 aq, 2 aq + 1: weights 8 aq .. + 7). A warp's
        //      32 lanes then read 8 rows x 4 column words: rows 880 B apart sit 4 banks
        //      apart, the quarters 1 bank apart, so the raw-tile loads are conflict-free
        //   B: (pair column, 8-wide chunk) jobs q = tid and tid + 256 of the slice (n_pad x 4 jobs)
        const int aq = lane >> 3, r1 = 16 * warp + (lane & 7);
        const int arow[2] = {r1, r1 + 8};
        const uint32_t grep = (uint32_t)(lane & (kGridReplicas - 1));
        const uint8_t* raw = smem + Smem::raw;
        int g = 0, i = 0;
        for (int ti = blockIdx.x; ti < n_tasks && !*abort_flag; ti += gridDim.x, ++i) {
            const Task t = p.tasks[ti];
            const int nn = t.n, n_pad = (nn + 15) & ~15;
            if (tid == 0 && ti + (int)gridDim.x < n_tasks) {   // the next task's tile, into L2 meanwhile
                const Task tn = p.tasks[ti + gridDim.x];
                prefetch_l2(p.base + (size_t)tn.expert * p.expert_stride + (size_t)tn.mt * kM * p.rb, tile_bytes);
            }
            const uint8_t* rowp[2] = {raw + (size_t)arow[0] * p.rb, raw + (size_t)arow[1] * p.rb};
            // pair tables of the task (epilogue) and this thread's B jobs
            if (tid < nn) {
                const PairInfo pi = p.pairs[t.n0 + tid];
                pair_exp[tid] = pi.exp;
                pair_dst[tid] = (float*)(p.dst + pi.dst_off);
            }
            const float* bx[2] = {nullptr, nullptr};
            float bs[2] = {0.f, 0.f};
            int bcol[2] = {-1, -1}, bch[2] = {0, 0};
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int q = tid + kProducers * u;
                if (q < n_pad * 4) {
                    bcol[u] = q >> 2;
                    bch[u] = q & 3;
                    if (bcol[u] < nn) {
                        const PairInfo pi = p.pairs[t.n0 + bcol[u]];
                        bx[u] = (const float*)(p.x + pi.x_off) + 8 * bch[u];
                        bs[u] = ldexpf(1.f, pi.exp);
                    }
                }
            }
            mbar_wait(rawbar, i & 1, p.err, abort_flag);   // on failure the abort flag is read below
            if (tid == 0) ++raw_waited;
            if (aq == 0) {
                // row scale: |w| <= |d| * 31 * 15 per super-block
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    float m = 0.f;
                    for (int j = 0; j < p.k / 256; ++j)
                        m = fmaxf(m, fabsf(f16_bits(*(const unsigned short*)(rowp[u] + j * 110))));
                    m *= 465.f;
                    int ex = 0;
                    if (m > 0.f && isfinite(m)) {
                        frexpf(m, &ex);
                        ex = max(-100, min(100, 14 - ex));
                    }
                    row_exp[arow[u]] = ex;
                }
            }
            producers_sync();   // row scales written; a uniform decision on the abort flag
            if (*abort_flag) break;
            const float rs[2] = {ldexpf(1.f, row_exp[arow[0]]), ldexpf(1.f, row_exp[arow[1]])};
            // B: the next slice's x is loaded while the current one is converted
            float4 xn[2][2];
#pragma unroll
            for (int u = 0; u < 2; ++u)
                if (bx[u]) {
                    xn[u][0] = __ldg((const float4*)bx[u]);
                    xn[u][1] = __ldg((const float4*)bx[u] + 1);
                }
            for (int kt = 0; kt < nk; ++kt, ++g) {
                const int s = g % kStages;
                if (g >= kStages) {   // one poller per warp
                    bool ok = true;
                    if (lane == 0) ok = mbar_wait(empty0 + 8 * s, ((g / kStages) - 1) & 1, p.err, abort_flag);
                    if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
                }
                uint8_t* st = smem + Smem::stage + s * kStageBytes;
                {   // A: weights 8 aq .. 8 aq + 7 (entries 2 aq, 2 aq + 1) of sub-block kt of rows arow[]
                    const int j = kt >> 3, ib = kt & 7;
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint8_t* bb = rowp[u] + j * 110;
                        const unsigned sc = (bb[106 + (ib >> 1)] >> (4 * (ib & 1))) & 15;
                        const float db = f16_bits(*(const unsigned short*)bb) * (float)(1 + 2 * sc) * rs[u];
                        const float dbc = -8388608.f * db;   // byte b -> float(2^23 + b) * db - 2^23 * db = b * db
                        const unsigned qh = bb[66 + ib];
                        const int c = aq;
                        const int r = arow[u];
                        const unsigned qs2 = *(const unsigned short*)(bb + 2 + 8 * ib + 2 * c);
                        const unsigned sg = bb[74 + 4 * ib + c];
                        float v[8];
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            const int e = 2 * c + q;
                            const unsigned idx = ((qs2 >> (8 * q)) & 255) | (((qh >> e) & 1) << 8);
                            const uint32_t gw = gtab[idx * kGridReplicas + grep];
#pragma unroll
                            for (int m = 0; m < 4; ++m) {
                                // bytes [grid byte m, 0, 0, 0x4B] = the float 2^23 + byte
                                const float magic = __uint_as_float(prmt(gw, 0x4B000000u, (uint32_t)m | 0x7540u));
                                const float val = fmaf(magic, db, dbc);
                                v[4 * q + m] = __uint_as_float(__float_as_uint(val) ^ (((sg >> (4 * q + m)) & 1u) << 31));
                            }
                        }
                        uint4 hi, lo;
                        split8(v, hi, lo);
                        const uint32_t off = chunk_off(r, c, kM);
                        *(uint4*)(st + off) = hi;
                        *(uint4*)(st + kAHalf + off) = lo;
                    }
                }
#pragma unroll
                for (int u = 0; u < 2; ++u) {   // B jobs
                    if (bcol[u] < 0) continue;
                    float v[8];
                    if (bx[u]) {
                        const float4 a0 = xn[u][0], a1 = xn[u][1];
                        if (kt + 1 < nk) {
                            xn[u][0] = __ldg((const float4*)(bx[u] + (kt + 1) * kKs));
                            xn[u][1] = __ldg((const float4*)(bx[u] + (kt + 1) * kKs) + 1);
                        }
                        v[0] = a0.x * bs[u]; v[1] = a0.y * bs[u]; v[2] = a0.z * bs[u]; v[3] = a0.w * bs[u];
                        v[4] = a1.x * bs[u]; v[5] = a1.y * bs[u]; v[6] = a1.z * bs[u]; v[7] = a1.w * bs[u];
                    } else {
#pragma unroll
                        for (int q = 0; q < 8; ++q) v[q] = 0.f;
                    }
                    uint4 hi, lo;
                    split8(v, hi, lo);
                    const uint32_t off = chunk_off(bcol[u], bch[u], kMaxN);
                    *(uint4*)(st + 2 * kAHalf + off) = hi;
                    *(uint4*)(st + 2 * kAHalf + kBHalf + off) = lo;
                }
                // the generic-proxy writes above are read by the tensor cores (async proxy);
                // one arrival per warp once all its lanes have fenced
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(full0 + 8 * s);
            }
            // ---- epilogue: warp w reads TMEM lanes 32 * (w & 3) .. + 31, columns (w >> 2) * 64 .. + 63
            producers_sync();   // row and pair tables of this task are written; the raw tile is consumed
            if (tid == 0 && ti + (int)gridDim.x < n_tasks && !*abort_flag) {
                issue_raw(ti + gridDim.x);
                ++raw_issued;
            }
            // warp-uniform: tcgen05.ld below is a whole-warp instruction
            const bool ok = __all_sync(0xffffffffu, mbar_wait(tfull, i & 1, p.err, abort_flag));
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            if (ok) {
                const int q = warp & 3, row = 32 * q + lane;
                const int grow = t.mt * kM + row;
                const int rexp = row_exp[row];
                for (int cc = (warp >> 2) * 64; cc < (warp >> 2) * 64 + 64 && cc < n_pad; cc += 16) {
                    float v[16];
                    tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)cc, v);
#pragma unroll
                    for (int u = 0; u < 16; ++u) {
                        const int c = cc + u;
                        if (c < nn) pair_dst[c][grow] = ldexpf(v[u], -(rexp + pair_exp[c]));
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            producers_sync();   // tables may be rewritten; the accumulator is free
            if (lane == 0) mbar_arrive(tempty);
            if (!ok) break;
        }
    }
    // never leave with a tile copy in flight
    if (tid == 0)
        for (; raw_waited < raw_issued; ++raw_waited)
            for (long long it = 0; it < kSpinLimit && !mbar_try_wait(rawbar, raw_waited & 1); ++it) {
            }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (warp == kProducers / 32) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kMaxN));
}

// ------------------------------------------------------------ grouping
// pairs p = (t, i), p = t * n_ids + i
struct GroupParams {
    sb_experts ex;
    int n_ids, n_tokens, n_experts, m_tiles;
    const uint8_t* x;
    size_t x_id_stride, x_token_stride;
    int x_rows, k;
    size_t dst_id_stride, dst_token_stride;
    int* counts;      // [n_experts]
    int* cursor;      // [n_experts]
    Task* tasks;      // tcgen05 tasks: experts with >= heavy pairs
    int* n_tasks;
    Task* mtasks;     // register-decode entries (experts with < heavy pairs, cut into groups of at
                      // most kGMaxPairs): {expert, -, first pair, pairs}; a task is (entry,
                      // 128-row block), task index = entry * m_tiles + block
    int* n_mtasks;    // entries * m_tiles
    int* mnext;       // the register-decode kernel's next task, [0] and [4] (zeroed by the plan)
    int heavy;
    int* order;       // [pairs] pair index in grouped order
    PairInfo* pairs;  // [pairs] grouped order
    int* err;
};

__device__ inline int pair_expert(const GroupParams& g, int pr) {
    const int t = pr / g.n_ids, i = pr % g.n_ids;
    int id = *(const int32_t*)((const uint8_t*)g.ex.ids + (size_t)t * g.ex.ids_token_stride +
                               (size_t)i * g.ex.ids_id_stride);
#if SABAH_SENTINEL == 1
    if (i == 0 && id >= 0 && id < g.n_experts) id = (id + 1) % g.n_experts;   // test-only build
#endif
    return id;
}

__global__ void k_group_count(const GroupParams g) {
    const int n = g.n_ids * g.n_tokens;
    for (int pr = blockIdx.x * blockDim.x + threadIdx.x; pr < n; pr += gridDim.x * blockDim.x) {
        const int e = pair_expert(g, pr);
        if (e < 0 || e >= g.n_experts) {
            if (g.err) atomicExch(g.err, SB_DERR_BAD_ID);
            continue;
        }
        atomicAdd(g.counts + e, 1);
    }
}

// one CTA of 1024 threads: exclusive scans of the counts and of the tasks per expert
__global__ void k_group_plan(const GroupParams g) {
    __shared__ int s_sum[1024], s_tsum[1024], s_msum[1024];
    const int E = g.n_experts, per = (E + 1023) / 1024;
    const int e0 = threadIdx.x * per, e1 = min(E, e0 + per);
    int c = 0, tc = 0, mc = 0;
    for (int e = e0; e < e1; ++e) {
        const int ce = g.counts[e];
        c += ce;
        if (ce >= g.heavy) tc += (ce + kMaxN - 1) / kMaxN * g.m_tiles;
        else mc += (ce + kGMaxPairs - 1) / kGMaxPairs;
    }
    s_sum[threadIdx.x] = c;
    s_tsum[threadIdx.x] = tc;
    s_msum[threadIdx.x] = mc;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {   // inclusive Hillis-Steele scans
        const int a = threadIdx.x >= off ? s_sum[threadIdx.x - off] : 0;
        const int b = threadIdx.x >= off ? s_tsum[threadIdx.x - off] : 0;
        const int m = threadIdx.x >= off ? s_msum[threadIdx.x - off] : 0;
        __syncthreads();
        s_sum[threadIdx.x] += a;
        s_tsum[threadIdx.x] += b;
        s_msum[threadIdx.x] += m;
        __syncthreads();
    }
    int pos = s_sum[threadIdx.x] - c, tpos = s_tsum[threadIdx.x] - tc, mpos = s_msum[threadIdx.x] - mc;
    for (int e = e0; e < e1; ++e) {
        const int ce = g.counts[e];
        g.cursor[e] = pos;
        if (ce >= g.heavy) {
            for (int n0 = 0; n0 < ce; n0 += kMaxN)
                for (int mt = 0; mt < g.m_tiles; ++mt) g.tasks[tpos++] = Task{e, mt, pos + n0, min(kMaxN, ce - n0)};
        } else {
            for (int n0 = 0; n0 < ce; n0 += kGMaxPairs) g.mtasks[mpos++] = Task{e, 0, pos + n0, min(kGMaxPairs, ce - n0)};
        }
        pos += ce;
    }
    if (threadIdx.x == 1023) {
        *g.n_tasks = s_tsum[1023];
        *g.n_mtasks = s_msum[1023] * g.m_tiles;
        g.mnext[0] = 0;
        g.mnext[4] = 0;   // the counter of a second run over the same plan (the block's up call)
    }
}

__global__ void k_group_scatter(const GroupParams g, uint8_t* dst, int rows) {
    const int n = g.n_ids * g.n_tokens;
    for (int pr = blockIdx.x * blockDim.x + threadIdx.x; pr < n; pr += gridDim.x * blockDim.x) {
        const int e = pair_expert(g, pr);
        if (e < 0 || e >= g.n_experts) {   // no expert: the pair's output row is NaN (error already set)
            float* d = (float*)(dst + (size_t)(pr / g.n_ids) * g.dst_token_stride + (size_t)(pr % g.n_ids) * g.dst_id_stride);
            for (int r = 0; r < rows; ++r) d[r] = __int_as_float(0x7fc00000);
            continue;
        }
        g.order[atomicAdd(g.cursor + e, 1)] = pr;
    }
}

// one warp per grouped position: x row offset, dst offset, x scale
__global__ void k_group_pairs(const GroupParams g) {
    const int n = g.n_ids * g.n_tokens;
    const int nw = gridDim.x * (blockDim.x / 32);
    const int lane = threadIdx.x & 31;
    for (int q = (blockIdx.x * blockDim.x + threadIdx.x) / 32; q < n; q += nw) {
        const int pr = g.order[q];
        if (pr < 0) continue;
        const int t = pr / g.n_ids, i = pr % g.n_ids;
        const long long xo = (long long)(t * g.x_token_stride + (i % g.x_rows) * g.x_id_stride);
        const float* xr = (const float*)(g.x + xo);
        float m = 0.f;
        for (int k = lane; k < g.k; k += 32) m = fmaxf(m, fabsf(xr[k]));
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) {
            int ex = 0;
            if (m > 0.f && isfinite(m)) {
                frexpf(m, &ex);
                ex = max(-100, min(100, 14 - ex));
            }
            g.pairs[q] = PairInfo{xo, (long long)(t * g.dst_token_stride + i * g.dst_id_stride), ex,
                                  t * g.x_rows + i % g.x_rows};
        }
    }
}

// Each x row (t, x_row) scaled by 2^exp (max -> [2^13, 2^14)) and split into
// fp16 hi / lo (truncated hi, exact; lo rounded), one warp per row.
__global__ void k_x_split(const uint8_t* x, size_t x_id_stride, size_t x_token_stride, int x_rows, int n_rows, int k,
                          __half* xh, __half* xl, int* xexp) {
    const int nw = gridDim.x * (blockDim.x / 32);
    const int lane = threadIdx.x & 31;
    for (int row = (blockIdx.x * blockDim.x + threadIdx.x) / 32; row < n_rows; row += nw) {
        const float* xr = (const float*)(x + (size_t)(row / x_rows) * x_token_stride + (size_t)(row % x_rows) * x_id_stride);
        float m = 0.f;
        for (int kk = lane; kk < k; kk += 32) m = fmaxf(m, fabsf(xr[kk]));
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        int ex = 0;
        if (m > 0.f && isfinite(m)) {
            frexpf(m, &ex);
            ex = max(-100, min(100, 14 - ex));
        }
        const float sc = ldexpf(1.f, ex);
        if (lane == 0) xexp[row] = ex;
        for (int kk = 2 * lane; kk < k; kk += 64) {
            const float a = xr[kk] * sc, b = xr[kk + 1] * sc;
            const float ah = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
            const float bh = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
            *(__half2*)(xh + (size_t)row * k + kk) = __floats2half2_rn(ah, bh);
            *(__half2*)(xl + (size_t)row * k + kk) = __floats2half2_rn(a - ah, b - bh);
        }
    }
}

// ------------------------------------------------------------ register-decode grouped kernel
// For experts with at most 8 routed pairs. A CTA task is (expert, 128-row
// block): the producer warp bulk-copies the pairs' x rows (fp16 hi and lo
// parts, split once per x row) and eight 16-row weight tiles into shared
// memory, its lanes issuing the copies side by side. Two consumer warps share
// a tile, one per half of its super-blocks (16 warps: enough independent work
// per SM to hide the latency of the shared loads and lookups). Each walks the
// IQ3_S sub-blocks of its half, decodes its A fragments once (mma.sync m16n8k16;
// the MMA's k slots {2c, 2c+1, 2c+8, 2c+9} are mapped to the 4 weights of grid
// entry c, placed as fp16 subnormals b * 2^-24 with their signs) and multiplies
// them with the pairs' x (the 8 pairs are the MMA's 8 columns); the sub-block's
// scale is applied to the fp32 partial sums. The second half's warp hands
// its sums to the first half's through shared memory (an mbarrier per tile),
// which adds them in that order and writes the rows. x and weights come from
// shared memory, so the K loop never waits on L2.
constexpr int kGW = 8;                       // 16-row tiles per task (one 128-row block)
constexpr int kGC = 2 * kGW;                 // consumer warps: (tile, half of the super-blocks)
constexpr int kGThreads = (kGC + 1) * 32;    // + the producer warp
constexpr int kGTile = 16 * 880;             // a 16-row tile at k <= 2048
constexpr int kGRep = 16;                    // grid-table replicas (lane % 16: at most 2-way bank conflicts)
constexpr int kGXRow = 2048 * 2 + 32;        // bytes per staged x row (fp16, padded against bank conflicts)

struct MmaSmem {
    static constexpr int grid = 0;                                   // [512][kGRep] u32
    static constexpr int xh = grid + 512 * kGRep * 4;                // [kGMaxPairs][kGXRow]
    static constexpr int xl = xh + kGMaxPairs * kGXRow;              // [kGMaxPairs][kGXRow]
    static constexpr int tiles = xl + kGMaxPairs * kGXRow;           // [kGW][kGTile]
    static constexpr int part = tiles + kGW * kGTile;                // [kGW][32 lanes][4] float: second-half sums
    static constexpr int bars = part + kGW * 32 * 16;                // xbar, free, tile[kGW], part[kGW]
    static constexpr int total = bars + (2 + 2 * kGW) * 8;
};
static_assert(MmaSmem::total <= 227 * 1024, "shared memory budget");
static_assert(MmaSmem::xh % 16 == 0 && MmaSmem::xl % 16 == 0 && MmaSmem::tiles % 16 == 0 && kGXRow % 16 == 0 &&
                  kGTile % 16 == 0,
              "bulk-copy alignment");

struct MmaParams {
    const uint8_t* base;
    size_t expert_stride;
    int rb, k, m_tiles;
    const Task* tasks;            // {expert, -, first pair, pairs}
    const int* n_tasks;           // entries * m_tiles
    int* next;                    // tasks are taken in order from this counter
    const PairInfo* pairs;
    const __half* xh;
    const __half* xl;
    const int* xexp;
    uint8_t* dst;
    int* err;
};

__device__ inline void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ inline void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__global__ void __launch_bounds__(kGThreads, 1) k_group_mma_iq3s(const MmaParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t* gtab = (uint32_t*)(smem + MmaSmem::grid);
    const uint32_t xbar = smem_u32(smem + MmaSmem::bars), freebar = xbar + 8, tbar0 = xbar + 16;
    const uint32_t pbar0 = tbar0 + 8 * kGW;   // per tile: the second half's sums are in
    volatile int* abort_flag = nullptr;
    __shared__ int s_abort;
    __shared__ int s_task;   // the current task (-1: none left), read after the x barrier
    for (int e = threadIdx.x; e < 512; e += kGThreads) {
        const uint32_t w = sb_iq3s_grid[e];
#pragma unroll
        for (int r = 0; r < kGRep; ++r) gtab[e * kGRep + r] = w;
    }
    if (threadIdx.x == 0) {
        s_abort = 0;
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(xbar));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(freebar), "r"(kGC));
        for (int w = 0; w < 2 * kGW; ++w) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tbar0 + 8 * w));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    abort_flag = &s_abort;
    const int n_tasks = *p.n_tasks;
    const uint32_t tile_bytes = (uint32_t)(16 * p.rb), xrow_bytes = (uint32_t)(p.k * 2);
    auto task_at = [&](int ti) {
        Task t = p.tasks[ti / p.m_tiles];
        t.mt = ti % p.m_tiles;
        return t;
    };

    if (warp == kGC) {
        // ---------------------------------------------------------- producer
        // Tasks come in order from a global counter, so CTAs that start late
        // (on SMs the tcgen05 kernel still held) take fewer. Lane 0 takes a task,
        // publishes it and sets the x barrier's byte count; then lanes j < n copy
        // pair j's hi part, lanes 8 + j its lo part, lanes 16 + w tile w. With no
        // task left, lane 0 publishes -1 and arrives on the x barrier alone.
        int i = 0, last = -1;
        bool drained = false;
        for (;; ++i) {
            // the consumers are done with the previous task's buffers
            if (!__all_sync(0xffffffffu, i == 0 || mbar_wait(freebar, (i - 1) & 1, p.err, abort_flag))) break;
            int ti = 0;
            if (lane == 0) ti = atomicAdd(p.next, 1);
            ti = __shfl_sync(0xffffffffu, ti, 0);
            if (ti >= n_tasks) {
                if (lane == 0) {
                    s_task = -1;
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(xbar) : "memory");
                }
                drained = true;   // every copy issued so far was consumed
                break;
            }
            const Task t = task_at(ti);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (lane == 0) {
                s_task = ti;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(xbar),
                             "r"(2u * xrow_bytes * (uint32_t)t.n)
                             : "memory");
            }
            __syncwarp();
            if (lane < 16 && (lane & 7) < t.n) {
                const int j = lane & 7;
                const int xr = p.pairs[t.n0 + j].xrow;
                const size_t o = (size_t)xr * p.k;
                if (lane < 8)
                    bulk_copy(smem_u32(smem + MmaSmem::xh + j * kGXRow), p.xh + o, xrow_bytes, xbar);
                else
                    bulk_copy(smem_u32(smem + MmaSmem::xl + j * kGXRow), p.xl + o, xrow_bytes, xbar);
            } else if (lane >= 16 && lane < 16 + kGW) {
                const int w = lane - 16;
                const uint8_t* blk = p.base + (size_t)t.expert * p.expert_stride + (size_t)t.mt * kGW * tile_bytes;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tbar0 + 8 * w),
                             "r"(tile_bytes)
                             : "memory");
                bulk_copy(smem_u32(smem + MmaSmem::tiles + w * kGTile), blk + (size_t)w * tile_bytes, tile_bytes,
                          tbar0 + 8 * w);
            } else if (lane == 31 && ti + (int)gridDim.x < n_tasks) {   // a task about one round on, into L2
                const Task tn = task_at(ti + gridDim.x);
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                                 p.base + (size_t)tn.expert * p.expert_stride + (size_t)tn.mt * kGW * tile_bytes),
                             "r"(kGW * tile_bytes)
                             : "memory");
            }
            last = i;
        }
        // never leave with copies in flight: after a give-up, the last task's copies have landed
        if (!drained && last >= 0 && lane == 0) {
            for (long long it = 0; it < kSpinLimit && !mbar_try_wait(xbar, last & 1); ++it) {
            }
            for (int w = 0; w < kGW; ++w)
                for (long long it = 0; it < kSpinLimit && !mbar_try_wait(tbar0 + 8 * w, last & 1); ++it) {
                }
        }
        // this kernel's stream successors also wait for the tcgen05 kernel's rows
        asm volatile("griddepcontrol.wait;" ::: "memory");
        return;
    }

    // -------------------------------------------------------------- consumers
    const int g = lane >> 2, c = lane & 3;
    const uint32_t grep = (uint32_t)(lane & (kGRep - 1));
    const int tw = warp & (kGW - 1), kh = warp / kGW;   // tile, half of the super-blocks
    const uint8_t* tile = smem + MmaSmem::tiles + tw * kGTile;
    float4* part = (float4*)(smem + MmaSmem::part) + tw * 32 + lane;
    const int nsb = p.k / 256, sb_mid = (nsb + 1) / 2;
    const int j_lo = kh ? sb_mid : 0, j_hi = kh ? nsb : sb_mid;
    const uint8_t* xhs = smem + MmaSmem::xh + g * kGXRow;   // this lane's pair column g
    const uint8_t* xls = smem + MmaSmem::xl + g * kGXRow;
    for (int i = 0;; ++i) {
        if (!__all_sync(0xffffffffu, mbar_wait(xbar, i & 1, p.err, abort_flag))) break;
        const int ti = *(volatile int*)&s_task;
        if (ti < 0) break;
        const Task t = task_at(ti);
        if (!__all_sync(0xffffffffu, mbar_wait(tbar0 + 8 * tw, i & 1, p.err, abort_flag))) break;
        const bool have = g < t.n;   // pair column g exists (else its B is zero)
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        // super-block by super-block: its scale d and 4 scale bytes are read
        // once, and its 8 sub-blocks are unrolled so their loads, lookups and
        // MMAs overlap (a warp needs independent work of its own to hide
        // latency: unrolling 4 sub-blocks instead, with the halves split by
        // sub-block, measured 7% slower on the whole prefill step)
        for (int j = j_lo; j < j_hi; ++j) {
            float d[2];
            uint32_t scw[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint8_t* rb = tile + (size_t)(g + 8 * h) * p.rb + j * 110;
                d[h] = __half2float(__ushort_as_half(*(const unsigned short*)rb)) * 16777216.f;   // 2^24: subnormal encoding
                scw[h] = (uint32_t)rb[106] | ((uint32_t)rb[107] << 8) | ((uint32_t)rb[108] << 16) |
                         ((uint32_t)rb[109] << 24);
            }
#pragma unroll
            for (int ib = 0; ib < 8; ++ib) {
                const int sb = 8 * j + ib;
                uint32_t a[2][2][2];   // [k16 half q][row h][reg]
                float db[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint8_t* rb = tile + (size_t)(g + 8 * h) * p.rb + j * 110;
                    const unsigned nib = (scw[h] >> (4 * ib)) & 15u;
                    db[h] = d[h] * (float)(1 + 2 * (int)nib);
                    const unsigned qh = rb[66 + ib];
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int e = 4 * q + c;
                        const uint32_t idx = rb[2 + 8 * ib + e] | (((qh >> e) & 1u) << 8);
                        const uint32_t gw = gtab[idx * kGRep + grep];
                        const uint32_t sg = (rb[74 + 4 * ib + (e >> 1)] >> (4 * (e & 1))) & 15u;
                        const uint32_t Z = (sg * 0x10204080u) & 0x80808080u;   // sign bit i -> bit 7 of byte i
                        a[q][h][0] = prmt(gw, Z, 0x5140);   // (w0, w1) as signed fp16 subnormals
                        a[q][h][1] = prmt(gw, Z, 0x7362);   // (w2, w3)
                    }
                }
                float dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int off = 2 * (32 * sb + 16 * q + 4 * c);
                    uint2 bh = make_uint2(0, 0), bl = make_uint2(0, 0);
                    if (have) {
                        bh = *(const uint2*)(xhs + off);
                        bl = *(const uint2*)(xls + off);
                    }
                    mma16816(dd, a[q][0][0], a[q][1][0], a[q][0][1], a[q][1][1], bh.x, bh.y);
                    mma16816(dd, a[q][0][0], a[q][1][0], a[q][0][1], a[q][1][1], bl.x, bl.y);
                }
                acc[0] = fmaf(db[0], dd[0], acc[0]);
                acc[1] = fmaf(db[0], dd[1], acc[1]);
                acc[2] = fmaf(db[1], dd[2], acc[2]);
                acc[3] = fmaf(db[1], dd[3], acc[3]);
            }
        }
        if (kh == 1) {
            // hand the second half's sums to the tile's first-half warp
            *part = make_float4(acc[0], acc[1], acc[2], acc[3]);
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(pbar0 + 8 * tw) : "memory");
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(freebar) : "memory");
            continue;
        }
        if (!__all_sync(0xffffffffu, mbar_wait(pbar0 + 8 * tw, i & 1, p.err, abort_flag))) break;
        {
            const float4 q = *part;
            acc[0] += q.x;
            acc[1] += q.y;
            acc[2] += q.z;
            acc[3] += q.w;
        }
        // D: (row g, pair 2c), (row g, pair 2c + 1), (row g + 8, pair 2c), (row g + 8, pair 2c + 1)
        const int row0 = (t.mt * kGW + tw) * 16;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int n = 2 * c + u;
            if (n >= t.n) continue;
            const PairInfo pi = p.pairs[t.n0 + n];
            float* d = (float*)(p.dst + pi.dst_off) + row0;
            const int ex = p.xexp[pi.xrow];
            d[g] = ldexpf(acc[u], -ex);
            d[g + 8] = ldexpf(acc[2 + u], -ex);
        }
        __syncwarp();   // every lane is done with the buffers
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(freebar) : "memory");
    }
    // this kernel's stream successors also wait for the tcgen05 kernel's rows
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ------------------------------------------------------------ host side
struct GroupScratch {
    void* mem = nullptr;
    size_t cap = 0;
};
GroupScratch g_gs;
bool g_attr_set = false;
int g_grid = 0;

bool prefill_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* v = std::getenv("SABAH_IQ3S_PREFILL");
        on = !(v && *v == '0');
    }
    return on != 0;
}

}  // namespace

// Experts with at least this many pairs go to the tcgen05 kernel; fewer are
// decoded in registers, 8 pairs per task. The register path decodes a weight
// ~4.5x faster but once per 8 pairs, the tcgen05 path once per 128. Measured
// on B200, 512-token Zipf(1.1) prefill: 2.01 / 1.71 / 1.75 / 1.81 ms per block
// at thresholds 9 / 25 / 33 / 49.
static int tc_min_pairs() {
    static int v = -1;
    if (v < 0) {
        const char* s = std::getenv("SABAH_IQ3S_TC_MIN_PAIRS");
        v = s && *s ? std::max(kGMaxPairs + 1, std::atoi(s)) : 25;
    }
    return v;
}

// Minimum (token, slot) pairs for the grouped path: below it the decode
// kernels, which stream each pair's tile once, are at least as fast.
int sb_prefill_min_pairs() {
    static int v = -1;
    if (v < 0) {
        const char* s = std::getenv("SABAH_IQ3S_PREFILL_MIN_PAIRS");
        v = s && *s ? std::max(1, std::atoi(s)) : 256;
    }
    return v;
}

namespace {
// The kernel parameters of the last grouped call, for a second run over the
// same plan (the fused block's up call: same ids, x, rows and k as its gate call)
struct LastPlan {
    GemmParams gp;
    MmaParams mp;
    bool valid = false;
} g_last_plan;
}  // namespace

int sb_try_mmid_iq3s_grouped(const sb_mmid_args& a, cudaStream_t st, bool force) {
    g_last_plan.valid = false;
    if (a.qt != SB_IQ3_S || !prefill_enabled() || a.ex.ptrs) return 0;
    const long long n_pairs = (long long)a.n_ids * a.n_tokens;
    if ((!force && n_pairs < sb_prefill_min_pairs()) || n_pairs < 1 || n_pairs > (1 << 24)) return 0;
    if (a.k % 256 || a.k > 2048 || a.rows % kM || a.ex.n_experts < 1 || a.ex.n_experts > 65536) return 0;
    const size_t rb = sb_row_bytes_of(SB_IQ3_S, a.k);
    if (a.row_stride != rb || ((uintptr_t)a.ex.base & 15) || a.ex.expert_stride % 16 || (kM * rb) % 16) return 0;
    if (((uintptr_t)a.x & 15) || a.x_id_stride % 16 || a.x_token_stride % 16) return 0;
    if (((uintptr_t)a.dst & 3) || a.dst_id_stride % 4 || a.dst_token_stride % 4) return 0;

    const int m_tiles = a.rows / kM;
    const long long max_tasks = (n_pairs / kMaxN + std::min<long long>(n_pairs, a.ex.n_experts) + 1) * m_tiles;
    const long long max_mtasks = n_pairs / kGMaxPairs + std::min<long long>(n_pairs, a.ex.n_experts) + 1;
    const long long n_xrows = (long long)a.n_tokens * a.x_rows;
    auto up256 = [](size_t b) { return (b + 255) & ~(size_t)255; };
    const size_t b_counts = up256((size_t)a.ex.n_experts * 4), b_cursor = b_counts;
    const size_t b_tasks = up256((size_t)max_tasks * sizeof(Task)), b_ntasks = 256;
    const size_t b_mtasks = up256((size_t)max_mtasks * sizeof(Task));
    const size_t b_order = up256((size_t)n_pairs * 4), b_pairs = up256((size_t)n_pairs * sizeof(PairInfo));
    const size_t b_xh = up256((size_t)n_xrows * a.k * 2), b_xexp = up256((size_t)n_xrows * 4);
    const size_t need = b_counts + b_cursor + b_tasks + b_ntasks + b_mtasks + b_order + b_pairs + 2 * b_xh + b_xexp;
    if (need > g_gs.cap) {
        if (g_gs.mem) {
            cudaDeviceSynchronize();   // no kernel of an earlier call may still use it
            cudaFree(g_gs.mem);
        }
        g_gs = GroupScratch{};
        if (!sb_cuda_ok(cudaMalloc(&g_gs.mem, need), "prefill scratch")) return -1;
        g_gs.cap = need;
    }
    uint8_t* b = (uint8_t*)g_gs.mem;
    GroupParams g{};
    g.ex = a.ex;
    g.n_ids = a.n_ids;
    g.n_tokens = a.n_tokens;
    g.n_experts = a.ex.n_experts;
    g.m_tiles = m_tiles;
    g.x = (const uint8_t*)a.x;
    g.x_id_stride = a.x_id_stride;
    g.x_token_stride = a.x_token_stride;
    g.x_rows = a.x_rows;
    g.k = a.k;
    g.dst_id_stride = a.dst_id_stride;
    g.dst_token_stride = a.dst_token_stride;
    g.counts = (int*)b;
    g.cursor = (int*)(b + b_counts);
    g.tasks = (Task*)(b + b_counts + b_cursor);
    uint8_t* q = b + b_counts + b_cursor + b_tasks;
    g.n_tasks = (int*)q;
    g.n_mtasks = (int*)(q + 16);
    g.mnext = (int*)(q + 32);
    q += b_ntasks;
    g.mtasks = (Task*)q;
    q += b_mtasks;
    g.order = (int*)q;
    q += b_order;
    g.pairs = (PairInfo*)q;
    q += b_pairs;
    __half* xh = (__half*)q;
    __half* xl = (__half*)(q + b_xh);
    int* xexp = (int*)(q + 2 * b_xh);
    g.heavy = tc_min_pairs();
    g.err = a.err;

    if (!g_attr_set) {
        if (!sb_cuda_ok(cudaFuncSetAttribute(k_prefill_iq3s, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::total),
                        "prefill smem attribute") ||
            !sb_cuda_ok(cudaFuncSetAttribute(k_group_mma_iq3s, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             MmaSmem::total),
                        "grouped mma smem attribute"))
            return -1;
        int dev = 0, sms = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        g_grid = std::max(1, sms);
        g_attr_set = true;
    }
    const int tslot = sb_timing_begin("prefill_iq3s", st);
    const int gblocks = (int)std::min<long long>((n_pairs + 255) / 256, 1024);
    if (!sb_cuda_ok(cudaMemsetAsync(g.counts, 0, b_counts, st), "prefill counts")) return -1;
    if (!sb_cuda_ok(cudaMemsetAsync(g.order, 0xff, b_order, st), "prefill order")) return -1;
    k_group_count<<<gblocks, 256, 0, st>>>(g);
    k_group_plan<<<1, 1024, 0, st>>>(g);
    k_group_scatter<<<gblocks, 256, 0, st>>>(g, (uint8_t*)a.dst, a.rows);
    k_group_pairs<<<(int)std::min<long long>((n_pairs + 7) / 8, 148LL * 8), 256, 0, st>>>(g);
    GemmParams gp{};
    gp.base = a.ex.base;
    gp.expert_stride = a.ex.expert_stride;
    gp.rb = (int)rb;
    gp.k = a.k;
    gp.rows = a.rows;
    gp.x = (const uint8_t*)a.x;
    gp.dst = (uint8_t*)a.dst;
    gp.tasks = g.tasks;
    gp.n_tasks = g.n_tasks;
    gp.pairs = g.pairs;
    gp.err = a.err;
    k_x_split<<<(int)std::min<long long>((n_xrows + 7) / 8, 148LL * 8), 256, 0, st>>>(
        (const uint8_t*)a.x, a.x_id_stride, a.x_token_stride, a.x_rows, (int)n_xrows, a.k, xh, xl, xexp);
    k_prefill_iq3s<<<g_grid, kThreads, Smem::total, st>>>(gp);   // experts with >= heavy pairs
    MmaParams mp{};
    mp.base = a.ex.base;
    mp.expert_stride = a.ex.expert_stride;
    mp.rb = (int)rb;
    mp.k = a.k;
    mp.m_tiles = m_tiles;
    mp.tasks = g.mtasks;
    mp.n_tasks = g.n_mtasks;
    mp.next = g.mnext;
    mp.pairs = g.pairs;
    mp.xh = xh;
    mp.xl = xl;
    mp.xexp = xexp;
    mp.dst = (uint8_t*)a.dst;
    mp.err = a.err;
    {   // the rest: a programmatic dependent of the tcgen05 kernel, whose SMs it
        // takes as that kernel's CTAs finish
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(g_grid);
        cfg.blockDim = dim3(kGThreads);
        cfg.dynamicSmemBytes = MmaSmem::total;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (!sb_cuda_ok(cudaLaunchKernelEx(&cfg, k_group_mma_iq3s, mp), "grouped mma launch")) return -1;
    }
    sb_timing_end(tslot, st);
    g_last_plan.gp = gp;
    g_last_plan.mp = mp;
    g_last_plan.valid = true;
    return sb_cuda_ok(cudaGetLastError(), "prefill launch") ? 1 : -1;
}

namespace {
// The last grouped call's two kernels again, over its plan and split x, for
// another bank of the same geometry into another output of the same strides.
// The plan's pair order, tasks and x rows depend only on the ids, x and the
// shapes, so none of the grouping kernels runs again.
int grouped_rerun(const uint8_t* base, size_t expert_stride, uint8_t* dst, cudaStream_t st) {
    if (!g_last_plan.valid || expert_stride != g_last_plan.gp.expert_stride) return 0;
    GemmParams gp = g_last_plan.gp;
    MmaParams mp = g_last_plan.mp;
    gp.base = mp.base = base;
    gp.dst = mp.dst = dst;
    mp.next = g_last_plan.mp.next + 4;   // the second counter, zeroed by the plan
    g_last_plan.valid = false;           // one rerun per plan: the second counter is spent
    const int tslot = sb_timing_begin("prefill_iq3s", st);
    k_prefill_iq3s<<<g_grid, kThreads, Smem::total, st>>>(gp);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(g_grid);
    cfg.blockDim = dim3(kGThreads);
    cfg.dynamicSmemBytes = MmaSmem::total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (!sb_cuda_ok(cudaLaunchKernelEx(&cfg, k_group_mma_iq3s, mp), "grouped mma launch")) return -1;
    sb_timing_end(tslot, st);
    return sb_cuda_ok(cudaGetLastError(), "prefill launch") ? 1 : -1;
}
}  // namespace

// ------------------------------------------------------------ the fused block, grouped
namespace {

// h = silu(g) * u, elementwise
__global__ void k_swiglu(const float* g, const float* u, float* h, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float gv = g[i];
        h[i] = gv / (1.f + expf(-gv)) * u[i];
    }
}

// out[t][i] = (accumulate ? out[t][i] : 0) + sum_e w[t][e] * y[t][e][i], slots in order
__global__ void k_combine(const float* y, const float* w, float* out, int n_tokens, int n_used, int d_model,
                          int accumulate) {
    const long long n = (long long)n_tokens * d_model;
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < n; q += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(q / d_model), i = (int)(q % d_model);
        float tot = 0.f;
        for (int e = 0; e < n_used; ++e)
            tot += w[(size_t)t * n_used + e] * y[((size_t)t * n_used + e) * d_model + i];
        out[q] = accumulate ? out[q] + tot : tot;
    }
}

struct BlockGroupedScratch {
    float* mem = nullptr;
    size_t cap = 0;   // floats
};
BlockGroupedScratch g_bgs;

// Whether the fused block runs grouped. SABAH_IQ3S_BLOCK_GROUPED_MIN fixes a
// pair threshold; by default a cost model chooses, fitted on B200 (2048 x 768
// IQ3_S experts, uniform routing, 64 and 512 experts, 1-1024 pairs): the
// one-launch path costs ~20 us plus ~1.1 us a pair with one slot per token
// (32-row down items) and ~1.4 us a pair otherwise; the grouped path ~145 us
// plus ~1.5 us per distinct expert and 8-pair task (refitted after the
// register-decode kernel moved to 16 warps and to the tcgen05 kernel's tail:
// 640 one-slot pairs over 512 experts take 691 us grouped, 698 us in one
// launch, and the whole expert-parallel step gains 7.6%), with the distinct experts of
// P uniformly routed pairs over E expected at E (1 - exp(-P / E)). The ids are
// on the device, so the expectation stands in for the count.
bool block_grouped_wins(long long pairs, int n_experts, int n_used) {
    static int v = -1;
    if (v < 0) {
        const char* s = std::getenv("SABAH_IQ3S_BLOCK_GROUPED_MIN");
        v = s && *s ? std::max(1, std::atoi(s)) : 0;
    }
    if (v > 0) return pairs >= v;
    const double P = (double)pairs, E = (double)std::max(1, n_experts);
    const double distinct = E * (1.0 - std::exp(-P / E));
    const double tasks = distinct * std::max(1.0, std::ceil(P / distinct / 8.0));
    return 145.0 + 1.5 * tasks < (n_used == 1 ? 20.0 + 1.1 * P : 1.4 * P);
}

}  // namespace

// Token t's input row xrows[t] of x into dst row t; a row index outside
// [0, n_xrows) gives a NaN row and SB_DERR_BAD_ID, as in the one-launch path.
__global__ void k_rows_gather(const float4* x, int n_xrows, const int32_t* xrows, int n, int k4, float4* dst, int* err) {
    const long long total = (long long)n * k4;
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < total; q += (long long)gridDim.x * blockDim.x) {
        const int i = (int)(q / k4), j = (int)(q % k4);
        const int r = __ldg(xrows + i);
        if (r < 0 || r >= n_xrows) {
            const float f = __int_as_float(0x7fc00000);
            if (err && j == 0) atomicExch(err, SB_DERR_BAD_ID);
            dst[q] = make_float4(f, f, f, f);
        } else {
            dst[q] = __ldg(x + (size_t)r * k4 + j);
        }
    }
}

int sb_block_iq3s_grouped(const sb_block_args& a, cudaStream_t st) {
    if (a.qt_gate != SB_IQ3_S || a.qt_up != SB_IQ3_S || a.qt_down != SB_IQ3_S || !prefill_enabled()) return 0;
    const long long slots = (long long)a.n_tokens * a.n_used;
    if (!block_grouped_wins(slots, a.gate.n_experts, a.n_used) || slots > (1 << 22)) return 0;
    if (a.gate.ptrs || a.up.ptrs || a.down.ptrs) return 0;
    if (a.d_model % 256 || a.ff % 256 || a.d_model > 2048 || a.ff > 2048 || a.d_model % kM || a.ff % kM) return 0;
    for (const sb_experts* e : {&a.gate, &a.up, &a.down})
        if (((uintptr_t)e->base & 15) || e->expert_stride % 16) return 0;
    if (((uintptr_t)a.x & 15) || ((uintptr_t)a.h & 15) || ((uintptr_t)a.out & 3)) return 0;

    // gathered inputs (token t reads row xrows[t]) are copied into place first
    const size_t gathered = a.xrows ? (size_t)a.n_tokens * a.d_model : 0;
    const size_t need = (size_t)slots * (2 * a.ff + a.d_model) + gathered;
    if (need > g_bgs.cap) {
        if (g_bgs.mem) {
            cudaDeviceSynchronize();   // no kernel of an earlier call may still use it
            cudaFree(g_bgs.mem);
        }
        g_bgs = BlockGroupedScratch{};
        if (!sb_cuda_ok(cudaMalloc(&g_bgs.mem, need * sizeof(float)), "grouped block scratch")) return -1;
        g_bgs.cap = need;
    }
    float* gout = g_bgs.mem;
    float* uout = gout + slots * a.ff;
    float* dout = uout + slots * a.ff;
    const float* x = a.x;
    if (a.xrows) {
        float* xg = dout + slots * a.d_model;
        const long long n4 = (long long)a.n_tokens * (a.d_model / 4);
        k_rows_gather<<<(int)std::min<long long>((n4 + 255) / 256, 148LL * 8), 256, 0, st>>>(
            (const float4*)a.x, a.n_xrows, a.xrows, a.n_tokens, a.d_model / 4, (float4*)xg, a.err);
        x = xg;
    }

    sb_mmid_args m{};
    m.row_stride = sb_row_bytes_of(SB_IQ3_S, a.d_model);
    m.x = x;
    m.x_id_stride = (size_t)a.d_model * 4;
    m.x_rows = 1;
    m.x_token_stride = (size_t)a.d_model * 4;
    m.n_ids = a.n_used;
    m.n_tokens = a.n_tokens;
    m.dst_id_stride = (size_t)a.ff * 4;
    m.dst_token_stride = (size_t)a.n_used * a.ff * 4;
    m.rows = a.ff;
    m.k = a.d_model;
    m.qt = SB_IQ3_S;
    m.err = a.err;
    m.ex = a.gate;
    m.dst = gout;
    if (sb_try_mmid_iq3s_grouped(m, st, true) != 1) return -1;
    // up: the gate call's plan and split x again (same ids, x and shapes)
    const int rerun = grouped_rerun(a.up.base, a.up.expert_stride, (uint8_t*)uout, st);
    if (rerun < 0) return -1;
    if (rerun == 0) {
        m.ex = a.up;
        m.dst = uout;
        if (sb_try_mmid_iq3s_grouped(m, st, true) != 1) return -1;
    }
    const long long nh = slots * a.ff;
    const int tslot = sb_timing_begin("block_grouped_elementwise", st);
    k_swiglu<<<(int)std::min<long long>((nh + 255) / 256, 148LL * 8), 256, 0, st>>>(gout, uout, a.h, nh);
    sb_timing_end(tslot, st);
    m.ex = a.down;
    m.row_stride = sb_row_bytes_of(SB_IQ3_S, a.ff);
    m.x = a.h;
    m.x_id_stride = (size_t)a.ff * 4;
    m.x_rows = a.n_used;
    m.x_token_stride = (size_t)a.n_used * a.ff * 4;
    m.dst = dout;
    m.dst_id_stride = (size_t)a.d_model * 4;
    m.dst_token_stride = (size_t)a.n_used * a.d_model * 4;
    m.rows = a.d_model;
    m.k = a.ff;
    if (sb_try_mmid_iq3s_grouped(m, st, true) != 1) return -1;
    const long long no = (long long)a.n_tokens * a.d_model;
    const int tslot2 = sb_timing_begin("block_grouped_elementwise", st);
    k_combine<<<(int)std::min<long long>((no + 255) / 256, 148LL * 8), 256, 0, st>>>(dout, a.w, a.out, a.n_tokens,
                                                                                     a.n_used, a.d_model, a.accumulate);
    sb_timing_end(tslot2, st);
    return sb_cuda_ok(cudaGetLastError(), "grouped block launch") ? 1 : -1;
}
