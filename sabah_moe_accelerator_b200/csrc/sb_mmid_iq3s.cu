// IQ3_S routed-expert matvec on sm_100a: decode on the CUDA cores, multiply-
// accumulate on the tensor cores.
//
// Decoding an IQ3_S weight costs more instructions than its 0.43 bytes take to
// stream from HBM, so the kernel is built around instructions per weight and
// latency hiding, not around FLOPs:
//
// * Work is a sequence of "items": one 16-row tile of one expert matrix (or,
//   for gate/up, the gate tile and the up tile of the same 16 rows). A
//   producer warp streams item tiles HBM -> shared memory with cp.async.bulk
//   into a ring of stages guarded by mbarriers, and publishes a descriptor
//   (expert validity, token, slot, row tile, x-set slot) next to each stage.
// * Item i is split over `wpt` consumer warps by groups of 4 sub-blocks (128
//   weights of a row); the 12 consumer warps work on 12 / wpt items at once and
//   never meet at a CTA barrier: the last warp to finish an item (a shared
//   counter) sums the warps' partial rows in fixed order and runs the epilogue,
//   so results are deterministic.
// * A thread decodes one grid entry (4 weights) of a row into two half2
//   registers: one LDS.32 from a 16-fold replicated copy of the 512-entry grid
//   (a warp's lookups hit distinct banks pairwise), then two PRMTs place the
//   grid bytes as fp16 subnormals b * 2^-24 with their sign bits. Those are the
//   A operand of mma.sync.m16n8k16 (f16 x f16 -> f32).
// * K is permuted so one MMA covers 4 sub-blocks: quad c owns sub-block c of
//   the group, and the 8 N columns of B hold x of sub-block n/2 split into
//   fp16 hi (n even) and lo (n odd) parts, zero outside that sub-block. After
//   the 8 MMAs of a group, D[row][2c] + D[row][2c+1] is the sub-block dot, so a
//   sub-block scale is applied once per 32 weights, and hi + lo keeps the
//   products fp32-grade (~1e-7 relative).
// * x is scaled per 32-element sub-block by a power of two (max -> [2^13, 2^14));
//   that scale and the 2^24 of the subnormal encoding are undone in fp32.
//
// Three kernels share the engine: MUL_MAT_ID (v2 contract), fused gate/up +
// SwiGLU, and down + top-k weighted combine (+ residual/accumulate).
// Launches use programmatic dependent launch: a kernel's prologue and weight
// prefetch overlap the previous kernel; activations and outputs are touched
// only after griddepcontrol.wait. Every wait is bounded; on timeout the CTA
// records an error, skips its remaining work and drains its copies.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "sb_kernels.h"
#include "sb_quant.cuh"

namespace {

constexpr int kConsumers = 12;                   // consumer warps
constexpr int kThreads = (kConsumers + 1) * 32;  // + one producer warp
constexpr int kReplicas = 16;
constexpr int kTableBytes = 512 * kReplicas * 4; // 32 KB
constexpr int kStageBytes = 14336;               // >= 16 rows x 880 B
constexpr int kStages = 9;
constexpr int kSets = 4;
constexpr int kRecBytes = 72;                    // per (group, step): 4 quads x (hi, lo) x 8 B + 8 B zeros
constexpr int kGroupBytes = 8 * kRecBytes + 16;  // 8 records + 4 per-sub-block inverse scales
constexpr int kSetBytes = 16 * kGroupBytes;      // k <= 2048
constexpr int kMaxWpt = 4;
constexpr int kMaxP = 4;                         // items in flight (kConsumers / wpt, wpt >= 3)
// Reduction slots: each in-flight position owns a ring of kRing slots. Warps of
// one position take its items in order, and a warp can run at most
// kStages / (ntile * P) <= 3 of the position's items ahead of the slowest one
// (the stage ring holds it back), so a ring of 4 is never overwritten while
// the last warp of an older item still reads it.
constexpr int kRing = 4;
constexpr int kRedSlots = kMaxP * kRing;
constexpr long long kSpinLimit = 1ll << 26;      // bounded waits

enum Mode { MODE_MMID = 0, MODE_GATE_UP = 1, MODE_DOWN = 2 };

struct Desc {
    int bad;       // 0 valid, else the device error code (the epilogue emits NaN)
    int slot;      // x-fragment set
    int t, e, rt;  // token, slot (expert choice), row tile
};

struct Smem {
    static constexpr int table = 0;
    static constexpr int stages = table + kTableBytes;
    static constexpr int sets = stages + kStages * kStageBytes;
    static constexpr int red = sets + kSets * kSetBytes;                  // [kRedSlots][kMaxWpt][32] floats
    static constexpr int desc = red + kRedSlots * kMaxWpt * 32 * 4;      // [kStages] Desc
    static constexpr int cnt = desc + kStages * (int)sizeof(Desc);       // [kRedSlots] ints
    static constexpr int abort_flag = cnt + kRedSlots * 4;
    static constexpr int bars = (abort_flag + 4 + 7) & ~7;                // full[kStages], empty[kStages]
    static constexpr int total = bars + 2 * kStages * 8;
};
static_assert(Smem::total <= 227 * 1024, "shared memory budget");

struct Params {
    int mode;
    int n_items;           // MMID / DOWN: tiles; GATE_UP: (gate, up) tile pairs
    int per_key;           // consecutive items sharing one x vector
    int wpt, gpw, P;       // warps per item, groups per warp, items in flight (12 / wpt)
    int k, rb, rtiles;     // row length, row bytes, 16-row tiles per matrix
    sb_mmid_args m;
    sb_block_args b;
    float* partial;        // DOWN: [T][n_used][d_model]
    int* counters;         // DOWN: [T][d_model / 16], self-resetting
    int* err;
};

// ---------------------------------------------------------------- PTX helpers
__device__ inline uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ inline void mbar_init(uint32_t bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ inline void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ inline void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
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
// then sets the abort flag and the device error word). Callers skip their work
// but keep taking part in every barrier, so nothing is left waiting.
__device__ inline bool mbar_wait(uint32_t bar, uint32_t parity, int* err, volatile int* abort_flag) {
    for (long long i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255 && *abort_flag) return false;
    }
    *abort_flag = 1;
    if (err) atomicExch(err, SB_DERR_TIMEOUT);
    return false;
}
__device__ inline void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ inline void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers * 32) : "memory"); }

__device__ inline uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ inline void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ inline uint32_t lds_u16(const uint8_t* p) { return *(const unsigned short*)p; }

// ---------------------------------------------------------------- items
__device__ inline const uint8_t* expert_ptr(const sb_experts& ex, int t, int i, int n_ids) {
    if (ex.ptrs) return (const uint8_t*)ex.ptrs[(size_t)t * n_ids + i];
    int id = *(const int32_t*)((const uint8_t*)ex.ids + (size_t)t * ex.ids_token_stride + (size_t)i * ex.ids_id_stride);
#if SABAH_SENTINEL == 1
    if (i == 0 && id >= 0 && id < ex.n_experts) id = (id + 1) % ex.n_experts;   // test-only build
#endif
    if (id < 0 || id >= ex.n_experts) return nullptr;
    return ex.base + (size_t)id * ex.expert_stride;
}

// 16-row tile `which` (0, or 1 = up for gate/up) of item `item`, its token/slot/row tile
__device__ inline const uint8_t* item_tile(const Params& p, int item, int which, int& t, int& e, int& rt) {
    const int rtiles = p.rtiles;
    rt = item % rtiles;
    const int si = item / rtiles;
    const uint8_t* base;
    if (p.mode == MODE_MMID) {
        t = si / p.m.n_ids;
        e = si % p.m.n_ids;
        base = expert_ptr(p.m.ex, t, e, p.m.n_ids);
        return base ? base + (size_t)rt * 16 * p.m.row_stride : nullptr;
    }
    t = si / p.b.n_used;
    e = si % p.b.n_used;
    const sb_experts& ex = p.mode == MODE_DOWN ? p.b.down : (which ? p.b.up : p.b.gate);
    base = expert_ptr(ex, t, e, p.b.n_used);
    return base ? base + (size_t)rt * 16 * p.rb : nullptr;
}

// the x vector of key (key = item / per_key)
__device__ inline const float* key_vector(const Params& p, int key) {
    if (p.mode == MODE_MMID) {
        // key = t * x_rows + x_row; items are ((t * n_ids + i) * rtiles + rt)
        int xt = key / p.m.x_rows, xr = key % p.m.x_rows;
#if SABAH_SENTINEL == 2
        if (p.m.x_rows > 1) xr = (xr + 1) % p.m.x_rows;   // test-only: wrong input row
#endif
#if SABAH_SENTINEL == 3
        xt = (xt + 1) % p.m.n_tokens;                     // test-only: wrong token
#endif
        return (const float*)((const uint8_t*)p.m.x + (size_t)xr * p.m.x_id_stride + (size_t)xt * p.m.x_token_stride);
    }
    if (p.mode == MODE_GATE_UP) return p.b.x + (size_t)key * p.b.d_model;
    return p.b.h + (size_t)key * p.b.ff;   // DOWN: key = t * n_used + e -> h[t][e]
}

// ---------------------------------------------------------------- x fragments
// B-operand set of vector x (length k): group q holds records (q, step s) with,
// for quad c, hi and lo half2 pairs of elements 32*(4q+c) + 4s .. +3 (scaled
// per sub-block), a zero pair, then the 4 inverse scales of its sub-blocks.
// Float4 f of x = entry f % 8 of sub-block f / 8. All consumer threads build.
__device__ void build_set(const float* x, int k, uint8_t* set) {
    const int nf = k / 4;
    for (int f = threadIdx.x; f < nf; f += kConsumers * 32) {
        const float4 v4 = __ldcg((const float4*)x + f);
        // the 8 float4 of sub-block j are 8 consecutive lanes: their max is the sub-block max
        float m = fmaxf(fmaxf(fabsf(v4.x), fabsf(v4.y)), fmaxf(fabsf(v4.z), fabsf(v4.w)));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        int ex = 0;
        if (m > 0.f && isfinite(m)) {
            frexpf(m, &ex);   // m = f * 2^ex, f in [0.5, 1)
            ex = max(-100, min(100, 14 - ex));
        }
        const float s = ldexpf(1.f, ex);
        const int j = f >> 3, st = f & 7, q = j >> 2, c = j & 3;
        const float v[4] = {v4.x * s, v4.y * s, v4.z * s, v4.w * s};
        __half hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            hi[i] = __float2half_rn(v[i]);
            lo[i] = __float2half_rn(v[i] - __half2float(hi[i]));
        }
        const __half2 h01 = __halves2half2(hi[0], hi[1]), h23 = __halves2half2(hi[2], hi[3]);
        const __half2 l01 = __halves2half2(lo[0], lo[1]), l23 = __halves2half2(lo[2], lo[3]);
        uint8_t* grp = set + q * kGroupBytes;
        uint2* rec = (uint2*)(grp + st * kRecBytes);
        rec[2 * c] = make_uint2(*(const uint32_t*)&h01, *(const uint32_t*)&h23);
        rec[2 * c + 1] = make_uint2(*(const uint32_t*)&l01, *(const uint32_t*)&l23);
        if (c == 0) rec[8] = make_uint2(0, 0);
        // 2^24 undoes the subnormal encoding of the weights, 1/s the x scale
        if (st == 0) ((float*)(grp + 8 * kRecBytes))[c] = 16777216.0f / s;
    }
}

// ---------------------------------------------------------------- decode core
// Decode groups [q0, q0 + NG) of a 16-row tile (NG interleaved MMA chains) and
// add their sub-block dots into acc[0] (row g) and acc[1] (row g + 8).
template <int NG>
__device__ inline void do_groups(const uint8_t* tile, int rb, int q0, const uint8_t* set, int boff,
                                 const uint32_t* table_lane, int g, int c, float (&acc)[2]) {
    uint32_t qs[NG][2][4], qh[NG][2], sgw[NG][2][4];
    float db[NG][2];
#pragma unroll
    for (int n = 0; n < NG; ++n) {
        const int q = q0 + n;
        const int jj = 4 * (q & 1) + c;   // sub-block inside the super-block
        const float inv = ((const float*)(set + q * kGroupBytes + 8 * kRecBytes))[c];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint8_t* bp = tile + (g + 8 * h) * rb + (q >> 1) * 110;
            const uint8_t* q8 = bp + 2 + 8 * jj;
#pragma unroll
            for (int w = 0; w < 4; ++w) qs[n][h][w] = lds_u16(q8 + 2 * w);
            qh[n][h] = (uint32_t)bp[66 + jj] << 8;
            const uint32_t sg = lds_u16(bp + 74 + 4 * jj) | (lds_u16(bp + 76 + 4 * jj) << 16);
            // sign nibble of entry s sits in the low or high nibble of sgw[s / 2]
            sgw[n][h][0] = sg;
            sgw[n][h][1] = sg >> 8;
            sgw[n][h][2] = sg >> 16;
            sgw[n][h][3] = sg >> 24;
            const int nib = (bp[106 + (jj >> 1)] >> (4 * (jj & 1))) & 15;
            db[n][h] = __half2float(__ushort_as_half((unsigned short)lds_u16(bp))) * (float)(1 + 2 * nib) * inv;
        }
    }
    float d[NG][4];
#pragma unroll
    for (int n = 0; n < NG; ++n) d[n][0] = d[n][1] = d[n][2] = d[n][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
#pragma unroll
        for (int n = 0; n < NG; ++n) {
            const uint2 bv = *(const uint2*)(set + (q0 + n) * kGroupBytes + s * kRecBytes + boff);
            uint32_t a[2][2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t w = qs[n][h][s >> 1];
                const uint32_t qsb = (s & 1) ? (w >> 8) : (w & 0xffu);
                const uint32_t idx = qsb | ((qh[n][h] >> s) & 0x100u);
                const uint32_t grid = table_lane[idx * kReplicas];
                // the 4 sign bits -> bit 7 of bytes 0..3 (nibble at bit 0 or 4 of sgw)
                const uint32_t nib = sgw[n][h][s >> 1] & ((s & 1) ? 0xF0u : 0x0Fu);
                const uint32_t Z = (nib * ((s & 1) ? 0x01020408u : 0x10204080u)) & 0x80808080u;
                a[h][0] = prmt(grid, Z, 0x5140);   // (e0, e1) as signed fp16 subnormals
                a[h][1] = prmt(grid, Z, 0x7362);   // (e2, e3)
            }
            mma16816(d[n], a[0][0], a[1][0], a[0][1], a[1][1], bv.x, bv.y);
        }
    }
#pragma unroll
    for (int n = 0; n < NG; ++n) {
        acc[0] = fmaf(db[n][0], d[n][0] + d[n][1], acc[0]);
        acc[1] = fmaf(db[n][1], d[n][2] + d[n][3], acc[1]);
    }
}

__device__ inline void decode_tile(const uint8_t* tile, int rb, int q0, int gpw, const uint8_t* set, int boff,
                                   const uint32_t* table_lane, int g, int c, float (&acc)[2]) {
    int q = q0;
    const int qe = q0 + gpw;
    for (; q + 2 <= qe; q += 2) do_groups<2>(tile, rb, q, set, boff, table_lane, g, c, acc);
    if (q < qe) do_groups<1>(tile, rb, q, set, boff, table_lane, g, c, acc);
}

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(kThreads, 1) k_iq3s(const Params p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bars = (uint64_t*)(smem + Smem::bars);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStages);
    volatile int* abort_flag = (volatile int*)(smem + Smem::abort_flag);
    Desc* descs = (Desc*)(smem + Smem::desc);
    const int ntile = p.mode == MODE_GATE_UP ? 2 : 1;   // tiles (stages) per item

    // let the next kernel on the stream begin its prologue as SMs free up
    asm volatile("griddepcontrol.launch_dependents;");

    // this CTA's item range
    const int i0 = (int)((long long)blockIdx.x * p.n_items / gridDim.x);
    const int i1 = (int)((long long)(blockIdx.x + 1) * p.n_items / gridDim.x);

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, p.wpt);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < kRedSlots) ((int*)(smem + Smem::cnt))[threadIdx.x] = 0;
    __syncthreads();

    if (warp == kConsumers) {
        // ------------------------------------------------------ producer
        if (lane == 0) {
            const uint32_t st0 = smem_u32(smem + Smem::stages);
            const uint32_t bytes = 16u * p.rb;
            int issued = 0;
            for (int item = i0; item < i1 && !*abort_flag; ++item) {
                for (int w = 0; w < ntile; ++w, ++issued) {
                    const int s = issued % kStages;
                    if (issued >= kStages &&
                        !mbar_wait(empty0 + 8 * s, ((issued / kStages) - 1) & 1, p.err, abort_flag))
                        break;
                    Desc d;
                    const uint8_t* src = item_tile(p, item, w, d.t, d.e, d.rt);
                    d.bad = !src ? SB_DERR_BAD_ID : ((uintptr_t)src & 15) ? SB_DERR_MISALIGNED : 0;
                    d.slot = (item / p.per_key) % kSets;
                    descs[s] = d;   // published by the arrive below (release)
                    if (!d.bad) {
                        mbar_expect_tx(full0 + 8 * s, bytes);
                        bulk_g2s(st0 + s * kStageBytes, src, bytes, full0 + 8 * s);
                    } else {
                        mbar_arrive(full0 + 8 * s);
                    }
                }
            }
            // never leave with copies in flight: the last use of every stage must land
            for (int n = std::max(0, issued - kStages); n < issued; ++n)
                for (long long i = 0; i < kSpinLimit && !mbar_try_wait(full0 + 8 * (n % kStages), (n / kStages) & 1);
                     ++i) {
                }
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    // replicated grid table: entry e, replica r at word e * kReplicas + r
    uint32_t* table = (uint32_t*)(smem + Smem::table);
    for (int e = threadIdx.x; e < 512; e += kConsumers * 32) {
        const uint32_t w = sb_iq3s_grid[e];
        uint4* dst = (uint4*)(table + e * kReplicas);
#pragma unroll
        for (int r = 0; r < kReplicas / 4; ++r) dst[r] = make_uint4(w, w, w, w);
    }
    // activations and outputs only after the previous kernel on the stream is done
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int g = lane >> 2, c = lane & 3;
    const uint32_t* table_lane = table + (lane & (kReplicas - 1));
    const int boff = (g >> 1) == c ? (2 * c + (g & 1)) * 8 : 64;
    const int pos = warp / p.wpt;   // which of the P items in flight
    const int wsub = warp % p.wpt;  // which part of the row
    float* red = (float*)(smem + Smem::red);
    int* cnt = (int*)(smem + Smem::cnt);
    const uint8_t* stages = smem + Smem::stages;
    uint8_t* sets = smem + Smem::sets;

    // Items are walked in chunks whose x vectors map to distinct set slots
    // (keys [kc * kSets, (kc + 1) * kSets)); sets are rebuilt at chunk starts.
    int item = i0;
    while (item < i1) {
        const int key0 = item / p.per_key;
        const int kc = key0 / kSets;
        const int chunk_end = min(i1, (kc + 1) * kSets * p.per_key);
        consumers_sync();   // all warps are done with the previous chunk's sets
        {
            const int k_last = (chunk_end - 1) / p.per_key;
            for (int key = key0; key <= k_last; ++key)
                build_set(key_vector(p, key), p.k, sets + (key % kSets) * kSetBytes);
        }
        consumers_sync();
        for (int it = item + pos, j = 0; it < chunk_end; it += p.P, ++j) {
            const int n_local = it - i0;               // item index in this CTA's sequence
            const int rslot = pos * kRing + (j % kRing);
            float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
            Desc d{};
            int bad = 0;
            for (int w = 0; w < ntile; ++w) {
                const int seq = n_local * ntile + w;    // stage sequence number
                const int s = seq % kStages;
                const bool landed = mbar_wait(full0 + 8 * s, (seq / kStages) & 1, p.err, abort_flag);
                d = descs[s];
                if (landed && !d.bad)
                    decode_tile(stages + s * kStageBytes, p.rb, wsub * p.gpw, p.gpw, sets + d.slot * kSetBytes, boff,
                                table_lane, g, c, acc[w]);
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * s);
                if (!bad) bad = landed ? d.bad : SB_DERR_TIMEOUT;
            }
            d.bad = bad;
            // this warp's rows: reduce the 4 quads, publish, count
#pragma unroll
            for (int w = 0; w < 2; ++w)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    acc[w][h] += __shfl_xor_sync(0xffffffffu, acc[w][h], 1);
                    acc[w][h] += __shfl_xor_sync(0xffffffffu, acc[w][h], 2);
                }
            float* rr = red + (rslot * kMaxWpt + wsub) * 32;
            if (c == 0) {
                rr[g] = acc[0][0];
                rr[g + 8] = acc[0][1];
                rr[16 + g] = acc[1][0];
                rr[16 + g + 8] = acc[1][1];
            }
            __threadfence_block();
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                last = atomicAdd(cnt + rslot, 1) == p.wpt - 1;
                if (last) cnt[rslot] = 0;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            __threadfence_block();
            // ---- epilogue (the last warp of the item), one row per lane
            if (lane < 16) {
                const float* r0 = red + rslot * kMaxWpt * 32;
                float v = 0.f, u = 0.f;
                for (int w = 0; w < p.wpt; ++w) {
                    v += r0[w * 32 + lane];
                    u += r0[w * 32 + 16 + lane];
                }
                if (d.bad) {
                    v = u = __int_as_float(0x7fc00000);
                    if (lane == 0 && p.err) atomicExch(p.err, d.bad);
                }
                const int row = d.rt * 16 + lane;
                if (p.mode == MODE_MMID) {
                    float* dst = (float*)((uint8_t*)p.m.dst + (size_t)d.t * p.m.dst_token_stride +
                                          (size_t)d.e * p.m.dst_id_stride);
                    dst[row] = v;
                } else if (p.mode == MODE_GATE_UP) {
                    p.b.h[((size_t)d.t * p.b.n_used + d.e) * p.b.ff + row] = v / (1.f + expf(-v)) * u;
                } else {
                    // DOWN: weighted partial; the last of the n_used slots of this
                    // row tile combines them in slot order
                    p.partial[((size_t)d.t * p.b.n_used + d.e) * p.b.d_model + row] =
                        p.b.w[(size_t)d.t * p.b.n_used + d.e] * v;
                    __threadfence();
                    __syncwarp(0x0000ffffu);
                    int fin = 0;
                    if (lane == 0) {
                        int* gc = p.counters + (size_t)d.t * p.rtiles + d.rt;
                        fin = atomicAdd(gc, 1) == p.b.n_used - 1;
                        if (fin) *gc = 0;
                    }
                    fin = __shfl_sync(0x0000ffffu, fin, 0);
                    if (fin) {
                        __threadfence();
                        float tot = 0.f;
                        for (int e = 0; e < p.b.n_used; ++e)
                            tot += __ldcg(p.partial + ((size_t)d.t * p.b.n_used + e) * p.b.d_model + row);
                        float* o = p.b.out + (size_t)d.t * p.b.d_model + row;
                        *o = p.b.accumulate ? *o + tot : tot;
                    }
                }
            }
        }
        item = chunk_end;
    }
}

// ------------------------------------------------------------------ host side
bool g_attr_set = false;
int g_num_sms = 0;

// split a row of k weights (G = k / 128 groups) over wpt warps, gpw groups each
bool plan_groups(int k, int& wpt, int& gpw) {
    if (k % 128 || k > 2048) return false;
    const int G = k / 128;
    for (int w : {4, 3}) {   // P = kConsumers / w <= kMaxP
        if (kConsumers % w == 0 && kConsumers / w <= kMaxP && G % w == 0 && G / w <= 8) {
            wpt = w;
            gpw = G / w;
            return true;
        }
    }
    return false;
}

int launch(Params& p, cudaStream_t st) {
    if (!g_attr_set) {
        if (!sb_cuda_ok(cudaFuncSetAttribute(k_iq3s, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::total),
                        "iq3s smem attribute"))
            return -1;
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        g_attr_set = true;
    }
    p.P = kConsumers / p.wpt;
    const int grid = std::max(1, std::min(p.n_items, g_num_sms));
    const int tslot = sb_timing_begin(p.mode == MODE_MMID ? "mmid_iq3s" : p.mode == MODE_GATE_UP ? "gate_up_iq3s"
                                                                                                  : "down_iq3s",
                                      st);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Smem::total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_iq3s, p);
    sb_timing_end(tslot, st);
    return sb_cuda_ok(e, "iq3s launch") ? 1 : -1;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// scratch of the down kernel: partial sums and self-resetting counters
float* g_partial = nullptr;
int* g_counters = nullptr;
size_t g_partial_cap = 0, g_counter_cap = 0;

bool down_scratch(size_t n_partial, size_t n_counters) {
    if (n_partial > g_partial_cap) {
        if (g_partial) cudaFree(g_partial);
        g_partial = nullptr;
        g_partial_cap = 0;
        if (!sb_cuda_ok(cudaMalloc(&g_partial, n_partial * sizeof(float)), "down scratch")) return false;
        g_partial_cap = n_partial;
    }
    if (n_counters > g_counter_cap) {
        if (g_counters) cudaFree(g_counters);
        g_counters = nullptr;
        g_counter_cap = 0;
        if (!sb_cuda_ok(cudaMalloc(&g_counters, n_counters * sizeof(int)), "down counters")) return false;
        if (!sb_cuda_ok(cudaMemset(g_counters, 0, n_counters * sizeof(int)), "down counters reset")) return false;
        g_counter_cap = n_counters;
    }
    return true;
}

bool fast_path_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* v = std::getenv("SABAH_IQ3S_MMA");
        on = !(v && *v == '0');
    }
    return on != 0;
}

}  // namespace

int sb_try_mmid_iq3s(const sb_mmid_args& a, cudaStream_t st) {
    if (a.qt != SB_IQ3_S || !fast_path_enabled()) return 0;
    int wpt, gpw;
    if (!plan_groups(a.k, wpt, gpw) || a.rows % 16) return 0;
    const size_t rb = sb_row_bytes_of(SB_IQ3_S, a.k);
    if (a.row_stride != rb || 16 * rb > (size_t)kStageBytes) return 0;
    if (!a.ex.ptrs && (!aligned16(a.ex.base) || a.ex.expert_stride % 16)) return 0;
    if (a.x_id_stride % 16 || a.x_token_stride % 16 || !aligned16(a.x)) return 0;
    const long long items = (long long)a.n_ids * a.n_tokens * (a.rows / 16);
    if (items > (1ll << 30)) return 0;
    Params p{};
    p.mode = MODE_MMID;
    p.rtiles = a.rows / 16;
    p.n_items = (int)items;
    p.per_key = a.x_rows == 1 ? a.n_ids * p.rtiles : p.rtiles;
    p.wpt = wpt;
    p.gpw = gpw;
    p.k = a.k;
    p.rb = (int)rb;
    p.m = a;
    p.err = a.err;
    return launch(p, st);
}

int sb_try_block_iq3s(const sb_block_args& a, cudaStream_t st) {
    if (a.qt_gate != SB_IQ3_S || a.qt_up != SB_IQ3_S || a.qt_down != SB_IQ3_S || !fast_path_enabled()) return 0;
    int wpt_g, gpw_g, wpt_d, gpw_d;
    if (!plan_groups(a.d_model, wpt_g, gpw_g) || !plan_groups(a.ff, wpt_d, gpw_d)) return 0;
    if (a.ff % 16 || a.d_model % 16) return 0;
    const size_t rbg = sb_row_bytes_of(SB_IQ3_S, a.d_model), rbd = sb_row_bytes_of(SB_IQ3_S, a.ff);
    if (16 * rbg > (size_t)kStageBytes || 16 * rbd > (size_t)kStageBytes) return 0;
    for (const sb_experts* e : {&a.gate, &a.up, &a.down})
        if (!e->ptrs && (!aligned16(e->base) || e->expert_stride % 16)) return 0;
    if (!aligned16(a.x) || !aligned16(a.h) || (a.d_model * 4) % 16 || (a.ff * 4) % 16) return 0;
    if (!down_scratch((size_t)a.n_tokens * a.n_used * a.d_model, (size_t)a.n_tokens * (a.d_model / 16))) return -1;

    Params p{};
    p.b = a;
    p.err = a.err;
    // gate + up + SwiGLU: items (t, e, row tile), each = gate tile + up tile
    p.mode = MODE_GATE_UP;
    p.rtiles = a.ff / 16;
    p.n_items = a.n_tokens * a.n_used * p.rtiles;
    p.per_key = a.n_used * p.rtiles;   // one x per token
    p.wpt = wpt_g;
    p.gpw = gpw_g;
    p.k = a.d_model;
    p.rb = (int)rbg;
    if (launch(p, st) < 0) return -1;
    // down + weighted combine: items (t, e, row tile)
    p.mode = MODE_DOWN;
    p.rtiles = a.d_model / 16;
    p.n_items = a.n_tokens * a.n_used * p.rtiles;
    p.per_key = p.rtiles;               // one h per (token, slot)
    p.wpt = wpt_d;
    p.gpw = gpw_d;
    p.k = a.ff;
    p.rb = (int)rbd;
    p.partial = g_partial;
    p.counters = g_counters;
    return launch(p, st);
}
