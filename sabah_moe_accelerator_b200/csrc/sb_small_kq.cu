// Small-batch routed block for the K-quants: Q4_K or Q6_K gate/up and down,
// 1-4 tokens, device-resident banks (sabah_moe_block_ids, and through it
// sabah_moe_decode). It restates the reference's fused block (k_gate_up /
// k_down, sabah/runtime/cuda/sabah_rt.cu:2725-2785) over its Q4_K / Q6_K
// sub-block decoders (sub32_q4_K, sabah_rt.cu:2462-2485; Q6_K as gguf-py
// quants.py:586).
//
// In a decode batch the tokens share experts (a Markov router keeps 8 of 10
// slots from one token to the next: 40 (token, slot) pairs meet about 16
// distinct experts per block), so each distinct expert's rows are decoded ONCE
// and multiplied with every token routed to it:
//
// * every CTA deduplicates the block's (token, slot) ids into distinct experts
//   (first-occurrence order), with the tokens of each;
// * gate/up (k_small<QT, true>): an item is 8 gate rows and the same 8 up rows
//   of one distinct expert, stacked as one 16-row MMA tile; the MMA's 8 columns
//   are the tokens' x in fp16 hi and lo parts; the epilogue writes
//   h = silu(g) * u for every (token, slot) pair routed to the expert;
// * down (k_small<QT, false>): an item is 16 down rows of one distinct expert;
//   the columns are the expert's tokens' h rows; the epilogue writes the
//   unweighted down rows of every pair; k_small_combine forms the slot-ordered
//   weighted sum (plus the residual with accumulate), as k_down does;
// * decode: a k-unit is 64 weights of a row; the 4-bit (Q4_K) or 6-bit (Q6_K)
//   values go into registers as fp16 subnormals q * 2^-24 (exact) and multiply
//   on mma.sync m16n8k16; each Q4_K sub-block (32 weights) or Q6_K scale group
//   (16 weights) gets its scale on the fp32 dot, with the affine part from x
//   sums staged beside x: d*sc*sum(q x) - dmin*m*sum(x) for Q4_K,
//   d*sc*(sum(q x) - 32*sum(x)) for Q6_K, the reference decoders' factoring.
// * x and h are staged per row as fp16 hi + lo after a power-of-two scale
//   (max into [2^13, 2^14)), so products keep ~22 bits, fp32-grade.
//
// Pipeline: a producer warp (8 issuing lanes) streams tiles into an 8-stage
// ring with cp.async.bulk and mbarriers; 16 consumer warps take an item's
// super-blocks, one each (8 warps per item at k = 2048, 3 at k = 768), and the
// last one to finish sums the partial rows in fixed order. Q4_K rows at k = 2048 are 1152 B, a
// multiple of 128, so the 8 rows an MMA reads at one offset would share banks;
// such tiles are copied row by row into a 1168-byte stride instead. Every wait
// is bounded; a CTA that gives up records SB_DERR_TIMEOUT and drains its copies.
#include <cuda_fp16.h>

#include <algorithm>
#include <climits>
#include <cstdlib>

#include "sb_iq3s_core.cuh"   // mbarrier, bulk-copy, PRMT and mma.sync helpers


namespace {

using namespace sb_iq3s;

constexpr int kW = 16;                         // consumer warps
constexpr int kCThreads = kW * 32;
constexpr int kThreads = kCThreads + 32;       // + the producer warp
constexpr int kStages = 8;                     // = kIssuers: lane l owns stage l
constexpr int kStageBytes = 16 * 1168;         // 16 padded Q4_K rows at k = 2048
constexpr int kMaxWpt = 8;                     // warps per item
constexpr int kMaxTok = 4;
constexpr int kMaxPairs = 64;
constexpr int kBArea = 8 * 2 * (1024 * 2 + 32);   // staged B rows: hi rows, then lo rows
constexpr int kLoOff = kBArea / 2;
constexpr int kMaxGroups = 512;                // staged 16-element groups (rows * k / 16)
static_assert(4 * (2048 * 2 + 32) <= kLoOff, "4 token rows at k = 2048");
static_assert(kStages == kIssuers, "a stage must always belong to the same producer lane");

struct Desc {
    int seq, bad, d, r;
};

struct Smem {
    static constexpr int stages = 0;
    static constexpr int barea = stages + kStages * kStageBytes;
    static constexpr int sums = barea + kBArea;                         // [rows][k / 16] float: sum of x
    static constexpr int inv = sums + kMaxGroups * 4;                   // [rows][k / 16] float: 2^-scale
    static constexpr int red = inv + kMaxGroups * 4;                    // [kStages][kMaxWpt][32] float2
    static constexpr int p_e = red + kStages * kMaxWpt * 32 * 8;        // [kMaxPairs] pair -> expert id (-1 bad)
    static constexpr int p_dist = p_e + kMaxPairs * 4;                  // [kMaxPairs] pair -> distinct index
    static constexpr int p_expert = p_dist + kMaxPairs * 4;             // [kMaxPairs] distinct -> expert id
    static constexpr int p_mask = p_expert + kMaxPairs * 4;             // [kMaxPairs] distinct -> token mask
    static constexpr int p_first = p_mask + kMaxPairs * 4;              // [kMaxPairs][kMaxTok] first pair
    static constexpr int misc = p_first + kMaxPairs * kMaxTok * 4;      // n_distinct, abort
    static constexpr int desc = misc + 16;                              // [kStages] Desc
    static constexpr int cnt = desc + kStages * (int)sizeof(Desc);      // [kStages] int
    static constexpr int bars = (cnt + kStages * 4 + 7) & ~7;           // full[kStages], empty[kStages]
    static constexpr int total = bars + 2 * kStages * 8;
};
static_assert(Smem::total <= 227 * 1024, "shared memory budget");
static_assert(kMaxGroups <= 2 * kCThreads, "stage_rows: at most 2 groups per thread");
static_assert(Smem::barea % 128 == 0 && kStageBytes % 128 == 0 && kLoOff % 128 == 0, "alignment");

struct SmallParams {
    const uint8_t* gate;
    const uint8_t* up;
    const uint8_t* down;
    size_t gu_stride, dn_stride;   // bytes between experts
    int rb, rs;                    // this phase's row bytes and staged row stride
    int k, rows_out;               // this phase's row length and output rows per expert
    const uint8_t* ids;
    size_t ids_id_stride, ids_token_stride;
    int n_experts, n_tokens, n_used, d_model, ff;
    const float* x;                // [T][d_model]
    float* h;                      // [T][n_used][ff]
    float* v;                      // [T][n_used][d_model] unweighted down rows
    int* err;
    // the down kernel of a block call: the call's gate/up kernel releases its
    // dependents only once its own grid dependency (the router ids' writer) is
    // done, so this kernel may read the ids before its own wait
    int ids_ready;
};

__device__ inline void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory"); }
// the routing plan is ready: the producer warp arrives, the consumers wait
__device__ inline void plan_arrive() { asm volatile("bar.arrive 2, %0;" ::"n"(kThreads) : "memory"); }
__device__ inline void plan_wait() { asm volatile("bar.sync 2, %0;" ::"n"(kThreads) : "memory"); }

// shared-memory loads at 32-bit shared addresses (explicit state space: a
// generic load would wait on the long scoreboard)
__device__ inline uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ inline uint32_t lds16(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ inline uint32_t lds16x2(uint32_t a) {   // 4 bytes at a 2-byte-aligned address
    return lds16(a) | (lds16(a + 2) << 16);
}
__device__ inline uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ inline float ldsf(uint32_t a) { return __uint_as_float(lds32(a)); }
// the j-th set bit (from bit 0) of a token mask
__device__ inline int nth_bit(unsigned m, int j) {
    for (int b = 0; b < kMaxTok; ++b)
        if ((m >> b) & 1u) {
            if (j == 0) return b;
            --j;
        }
    return 0;
}

// 4 bytes (q0..q3, each < 256) -> fp16 subnormal pairs (q0, q1), (q2, q3)
__device__ inline void to_f16(uint32_t q, uint32_t& lo, uint32_t& hi) {
    lo = prmt(q, 0u, 0x4140);
    hi = prmt(q, 0u, 0x4342);
}

// ------------------------------------------------------------ the routing plan
// Built by one warp: pairs p = t * n_used + i. A pair with an id outside
// [0, n_experts) sets the error word and belongs to no expert.
__device__ void build_plan(const SmallParams& p, uint8_t* smem) {
    int* s_e = (int*)(smem + Smem::p_e);
    int* s_dist = (int*)(smem + Smem::p_dist);
    int* s_expert = (int*)(smem + Smem::p_expert);
    int* s_mask = (int*)(smem + Smem::p_mask);
    int* s_first = (int*)(smem + Smem::p_first);
    const int lane = threadIdx.x & 31;
    const int n = p.n_tokens * p.n_used;
    int e[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int q = lane + 32 * u;
        e[u] = -1;
        if (q < n) {
            const int t = q / p.n_used, i = q % p.n_used;
            int id = *(const int32_t*)(p.ids + (size_t)t * p.ids_token_stride + (size_t)i * p.ids_id_stride);
#if SABAH_SENTINEL == 1
            if (i == 0 && id >= 0 && id < p.n_experts) id = (id + 1) % p.n_experts;   // test-only build
#endif
            if (id < 0 || id >= p.n_experts) {
                if (p.err) atomicExch(p.err, SB_DERR_BAD_ID);
                id = -1;
            }
            e[u] = id;
        }
        s_e[q] = e[u];
        s_mask[q] = 0;
#pragma unroll
        for (int j = 0; j < kMaxTok; ++j) s_first[q * kMaxTok + j] = INT_MAX;
    }
    __syncwarp();
    int fq[2];   // the first pair with the same expert
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int q = lane + 32 * u;
        fq[u] = q;
        if (e[u] >= 0)
            for (int r = 0; r < q; ++r)
                if (s_e[r] == e[u]) {
                    fq[u] = r;
                    break;
                }
    }
    const unsigned b0 = __ballot_sync(0xffffffffu, e[0] >= 0 && fq[0] == lane);
    const unsigned b1 = __ballot_sync(0xffffffffu, e[1] >= 0 && fq[1] == lane + 32);
    const unsigned lt = (1u << lane) - 1u;
    if (e[0] >= 0 && fq[0] == lane) {
        const int dd = __popc(b0 & lt);
        s_dist[lane] = dd;
        s_expert[dd] = e[0];
    }
    if (e[1] >= 0 && fq[1] == lane + 32) {
        const int dd = __popc(b0) + __popc(b1 & lt);
        s_dist[lane + 32] = dd;
        s_expert[dd] = e[1];
    }
    __syncwarp();
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int q = lane + 32 * u;
        if (e[u] < 0) s_dist[q] = -1;
        else if (fq[u] != q) s_dist[q] = s_dist[fq[u]];
    }
    __syncwarp();
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int q = lane + 32 * u;
        if (q < n && e[u] >= 0) {
            const int dd = s_dist[q], t = q / p.n_used;
            atomicOr(s_mask + dd, 1 << t);
            atomicMin(s_first + dd * kMaxTok + t, q);
        }
    }
    if (lane == 0) ((int*)(smem + Smem::misc))[0] = __popc(b0) + __popc(b1);
    __syncwarp();
}

// ------------------------------------------------------------ B staging
// n_rows rows of k fp32 values (row r from src(r), nullptr = zeros) into the B
// area as fp16 hi + lo. Each 16-element group is scaled by its own power of
// two (max into [2^13, 2^14)), whose inverse goes to inv[], and its plain sum
// to sums[]. One group per consumer thread, one pass; ends with
// consumers_sync. n_rows * k / 16 <= kMaxGroups.
template <class Src>
__device__ void stage_rows(uint8_t* smem, int n_rows, int k, Src src) {
    const int gi = threadIdx.x;
    const int gpr = k / 16, ng = n_rows * gpr;
    if (gi < ng) {
        const int row = gi / gpr, g16 = gi % gpr;
        const float* s = src(row);
        float4 v[4];
        float m = 0.f, sum = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[j] = s ? __ldcg((const float4*)(s + 16 * g16) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
            sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        }
        int ex = 0;
        if (m > 0.f && isfinite(m)) {
            frexpf(m, &ex);   // m = f * 2^ex, f in [0.5, 1)
            ex = max(-100, min(100, 14 - ex));
        }
        const float sc = ldexpf(1.f, ex);
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 q = v[j >> 1];
            const float a = ((j & 1) ? q.z : q.x) * sc, b = ((j & 1) ? q.w : q.y) * sc;
            const float ah = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
            const float bh = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
            const __half2 hh = __floats2half2_rn(ah, bh), ll = __floats2half2_rn(a - ah, b - bh);
            hw[j] = *(const uint32_t*)&hh;
            lw[j] = *(const uint32_t*)&ll;
        }
        uint8_t* hrow = smem + Smem::barea + row * (2 * k + 32) + 32 * g16;
        *(uint4*)hrow = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *(uint4*)(hrow + 16) = make_uint4(hw[4], hw[5], hw[6], hw[7]);
        *(uint4*)(hrow + kLoOff) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        *(uint4*)(hrow + kLoOff + 16) = make_uint4(lw[4], lw[5], lw[6], lw[7]);
        ((float*)(smem + Smem::sums))[gi] = sum;
        ((float*)(smem + Smem::inv))[gi] = ldexpf(1.f, -ex);
    }
    consumers_sync();
}

// ------------------------------------------------------------ decode
// One super-block (256 weights) of rows g and g + 8 of a tile, times this
// lane's B column; acc[h] collects row g + 8h of column pair c. bcol: this
// lane's column in the hi or lo B rows (byte address of element 0); sums: the
// scaled 16-element sums of column c. The super-block header is read once and
// its 4 k-units of 64 weights are unrolled, so every scale index is a constant.
template <int QT>
struct KQ;

template <>
struct KQ<SB_Q4_K> {
    // k-unit i: quant bytes 32i .. 32i + 31; low nibbles are sub-block 2i,
    // high nibbles sub-block 2i + 1
    __device__ static void superblock(uint32_t tile, int rs, int sbk, int g, int c, uint32_t bcol, bool have,
                                      uint32_t sums, uint32_t inv, float (&acc)[2]) {
        const uint32_t b[2] = {tile + (uint32_t)(g * rs + sbk * 144), tile + (uint32_t)((g + 8) * rs + sbk * 144)};
        float d[2], dmin[2];
        uint32_t W[2][3];   // the 12 scale bytes (ggml's get_scale_min_k4 packing, as sb_kscale)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t dm = lds32(b[h]);
            d[h] = __half2float(__ushort_as_half((unsigned short)(dm & 0xFFFF))) * 16777216.0f;   // 2^24: subnormal A
            dmin[h] = __half2float(__ushort_as_half((unsigned short)(dm >> 16)));
            W[h][0] = lds32(b[h] + 4);
            W[h][1] = lds32(b[h] + 8);
            W[h][2] = lds32(b[h] + 12);
        }
        const uint32_t bx = bcol + 2 * (sbk * 256 + 4 * c);
        const uint32_t sx = sums + 4 * sbk * 16, ix = inv + 4 * sbk * 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t w[2][2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                w[h][0] = lds32(b[h] + 16 + 32 * i + 4 * c);
                w[h][1] = lds32(b[h] + 16 + 32 * i + 16 + 4 * c);
            }
#pragma unroll
            for (int s = 0; s < 2; ++s) {   // sub-block j = 2i + s, elements 64i + 32s ..
                const int j = 2 * i + s;
                float dd[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};   // per 16-element half
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const uint32_t qg = s ? (w[0][half] >> 4) & 0x0F0F0F0Fu : w[0][half] & 0x0F0F0F0Fu;
                    const uint32_t q8 = s ? (w[1][half] >> 4) & 0x0F0F0F0Fu : w[1][half] & 0x0F0F0F0Fu;
                    uint32_t a0, a2, a1, a3;
                    to_f16(qg, a0, a2);
                    to_f16(q8, a1, a3);
                    uint2 bv = make_uint2(0u, 0u);
                    if (have) bv = lds64(bx + 2 * (64 * i + 32 * s + 16 * half));
                    mma16816(dd[half], a0, a1, a2, a3, bv.x, bv.y);
                }
                const int gq = 4 * i + 2 * s;   // the sub-block's two 16-element groups
                const float xs = ldsf(sx + 4 * gq) + ldsf(sx + 4 * gq + 4), i0 = ldsf(ix + 4 * gq), i1 = ldsf(ix + 4 * gq + 4);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    int sc, mn;
                    if (j < 4) {
                        sc = (W[h][0] >> (8 * j)) & 63;
                        mn = (W[h][1] >> (8 * j)) & 63;
                    } else {
                        const uint32_t b8 = (W[h][2] >> (8 * (j - 4))) & 0xFF;   // byte j + 4
                        sc = (b8 & 15) | (((W[h][0] >> (8 * (j - 4) + 6)) & 3) << 4);
                        mn = (b8 >> 4) | (((W[h][1] >> (8 * (j - 4) + 6)) & 3) << 4);
                    }
                    const float s0 = sb_mul(d[h], (float)sc);
                    const float off = -sb_mul(dmin[h], (float)mn);
                    const float dot = fmaf(dd[0][2 * h] + dd[0][2 * h + 1], i0, (dd[1][2 * h] + dd[1][2 * h + 1]) * i1);
                    acc[h] = fmaf(off, xs, fmaf(s0, dot, acc[h]));
                }
            }
        }
    }
};

template <>
struct KQ<SB_Q6_K> {
    // k-unit (hh, H): 128-weight half hh, 16-weight column half H; quadrants
    // p = 0..3 are weights 128hh + 32p + 16H + l, one scale group each
    __device__ static void superblock(uint32_t tile, int rs, int sbk, int g, int c, uint32_t bcol, bool have,
                                      uint32_t sums, uint32_t inv, float (&acc)[2]) {
        const uint32_t b[2] = {tile + (uint32_t)(g * rs + sbk * 210), tile + (uint32_t)((g + 8) * rs + sbk * 210)};
        float d[2];
        uint32_t SW[2][4];   // the 16 int8 scales
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            d[h] = __half2float(__ushort_as_half((unsigned short)lds16(b[h] + 208)));
#pragma unroll
            for (int q = 0; q < 4; ++q) SW[h][q] = lds16x2(b[h] + 192 + 4 * q);
        }
        const uint32_t bx = bcol + 2 * (sbk * 256 + 4 * c);
        const uint32_t sx = sums + 4 * sbk * 16, ix = inv + 4 * sbk * 16;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int hh = u >> 1, H = u & 1;
            uint32_t q[2][4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t qa = lds16x2(b[h] + 64 * hh + 16 * H + 4 * c);
                const uint32_t qb = lds16x2(b[h] + 64 * hh + 32 + 16 * H + 4 * c);
                const uint32_t qh = lds16x2(b[h] + 128 + 32 * hh + 16 * H + 4 * c);
                q[h][0] = (qa & 0x0F0F0F0Fu) | ((qh << 4) & 0x30303030u);
                q[h][1] = (qb & 0x0F0F0F0Fu) | ((qh << 2) & 0x30303030u);
                q[h][2] = ((qa >> 4) & 0x0F0F0F0Fu) | (qh & 0x30303030u);
                q[h][3] = ((qb >> 4) & 0x0F0F0F0Fu) | ((qh >> 2) & 0x30303030u);
            }
#pragma unroll
            for (int pq = 0; pq < 4; ++pq) {
                const int e = 128 * hh + 32 * pq + 16 * H;   // group's first element in the super-block
                uint32_t a0, a2, a1, a3;
                to_f16(q[0][pq], a0, a2);
                to_f16(q[1][pq], a1, a3);
                uint2 bv = make_uint2(0u, 0u);
                if (have) bv = lds64(bx + 2 * e);
                float dd[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(dd, a0, a1, a2, a3, bv.x, bv.y);
                const float xs = 32.f * ldsf(sx + 4 * (e >> 4)), iv = ldsf(ix + 4 * (e >> 4)) * 16777216.0f;   // 2^24: subnormal A
                const int idx = 8 * hh + 2 * pq + H;   // the group's scale: a constant after unrolling
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const float sc = (float)(int8_t)((SW[h][idx >> 2] >> (8 * (idx & 3))) & 0xFF);
                    acc[h] = fmaf(sb_mul(d[h], sc), fmaf(dd[2 * h] + dd[2 * h + 1], iv, -xs), acc[h]);
                }
            }
        }
    }
};

// ------------------------------------------------------------ the kernel
template <int QT, bool GU>
__global__ void __launch_bounds__(kThreads, 1) k_small(const __grid_constant__ SmallParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bars = (uint64_t*)(smem + Smem::bars);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStages);
    volatile int* abort_flag = (volatile int*)(smem + Smem::misc + 4);
    Desc* descs = (Desc*)(smem + Smem::desc);
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);   // one release per item, by its last warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < kStages) {
        ((int*)(smem + Smem::cnt))[threadIdx.x] = 0;
        descs[threadIdx.x].seq = -1;
    }
    __syncthreads();
    // programmatic dependent launch: the next kernel on the stream may start its
    // prologue (barrier set-up) as SMs free up. Everything this kernel reads
    // that an earlier kernel may write (router ids, x, h, v), and every global
    // write, comes after griddepcontrol.wait. The gate/up kernel releases its
    // dependents only after that wait, so the block's down kernel (ids_ready)
    // builds its routing plan from final ids while gate/up still runs.
    if (!GU && p.ids_ready) {
        asm volatile("griddepcontrol.launch_dependents;");
        if (warp == kW) {
            build_plan(p, smem);
            plan_arrive();
        }
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (warp != kW) plan_wait();
    } else {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;");
        if (warp == kW) {
            build_plan(p, smem);
            plan_arrive();
        } else {
            if (GU)   // the tokens' x, rows 0..T-1
                stage_rows(smem, kMaxTok, p.k,
                           [&](int r) { return r < p.n_tokens ? p.x + (size_t)r * p.d_model : nullptr; });
            plan_wait();
        }
    }

    const int nd = ((const int*)(smem + Smem::misc))[0];
    const int R = p.rows_out / (GU ? 8 : 16);   // items per distinct expert
    const int n_items = nd * R;
    const int i0 = (int)((long long)blockIdx.x * n_items / gridDim.x);
    const int i1 = (int)((long long)(blockIdx.x + 1) * n_items / gridDim.x);
    const int* s_expert = (const int*)(smem + Smem::p_expert);
    // down: experts per chunk of staged h rows (4 rows each)
    const int cpe = GU ? 1 << 20 : (p.k <= 1024 ? 2 : 1);

    if (warp == kW) {
        // ---------------------------------------------------------- producer
        if (lane < kIssuers) {
            const uint32_t st0 = smem_u32(smem + Smem::stages);
            const bool rowwise = p.rs != p.rb;
            int last = -1;
            for (int it = i0; it < i1; ++it) {
                const int n = it - i0;
                if (n % kIssuers != lane) continue;
                if (*abort_flag) break;
                const int s = n % kStages;
                if (n >= kStages && !mbar_wait(empty0 + 8 * s, ((n / kStages) - 1) & 1, p.err, abort_flag)) break;
                Desc d;
                d.d = it / R;
                d.r = it % R;
                const size_t e = (size_t)s_expert[d.d];
                d.bad = 0;
                d.seq = -1;
                descs[s] = d;
                __threadfence_block();
                *(volatile int*)&descs[s].seq = n;   // the stage's previous tile is released
                const uint32_t dst = st0 + s * kStageBytes;
                const uint32_t rows_b = 16u * (uint32_t)p.rb;
                mbar_expect_tx(full0 + 8 * s, rows_b);
                if (GU) {
                    const uint8_t* gsrc = p.gate + e * p.gu_stride + (size_t)(8 * d.r) * p.rb;
                    const uint8_t* usrc = p.up + e * p.gu_stride + (size_t)(8 * d.r) * p.rb;
                    if (!rowwise) {
                        bulk_g2s(dst, gsrc, rows_b / 2, full0 + 8 * s);
                        bulk_g2s(dst + 8u * p.rb, usrc, rows_b / 2, full0 + 8 * s);
                    } else {
                        for (int r = 0; r < 8; ++r) {
                            bulk_g2s(dst + r * p.rs, gsrc + (size_t)r * p.rb, p.rb, full0 + 8 * s);
                            bulk_g2s(dst + (8 + r) * p.rs, usrc + (size_t)r * p.rb, p.rb, full0 + 8 * s);
                        }
                    }
                } else {
                    const uint8_t* src = p.down + e * p.dn_stride + (size_t)(16 * d.r) * p.rb;
                    if (!rowwise) {
                        bulk_g2s(dst, src, rows_b, full0 + 8 * s);
                    } else {
                        for (int r = 0; r < 16; ++r)
                            bulk_g2s(dst + r * p.rs, src + (size_t)r * p.rb, p.rb, full0 + 8 * s);
                    }
                }
                last = n;
            }
            // never leave with a copy in flight
            if (last >= 0)
                for (long long i = 0; i < kSpinLimit && !mbar_try_wait(full0 + 8 * (last % kStages),
                                                                       (last / kStages) & 1); ++i) {
                }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    const int g = lane >> 2, c = lane & 3;
    // one super-block per warp: k / 256 warps per item (<= 8), P items at once
    const int wpt = p.k / 256;
    const int P = kW / wpt, pos = warp / wpt, wsub = warp % wpt;
    const int* s_dist = (const int*)(smem + Smem::p_dist);
    const int* s_mask = (const int*)(smem + Smem::p_mask);
    const int* s_first = (const int*)(smem + Smem::p_first);
    const float* sums = (const float*)(smem + Smem::sums);
    const float* invs = (const float*)(smem + Smem::inv);
    float2* red = (float2*)(smem + Smem::red);
    int* cnt = (int*)(smem + Smem::cnt);
    const int n_pairs = p.n_tokens * p.n_used;
    const int stride = 2 * p.k + 32;
    const int gpr = p.k / 16;
    int seq = 0;
    bool first_chunk = true;
    for (int d0 = i0 < i1 ? i0 / R : 0; i0 < i1 && d0 * R < i1; d0 += cpe) {
        const int cs = max(i0, d0 * R), ce = min(i1, (d0 + cpe) * R);
        if (!GU) {
            if (!first_chunk) consumers_sync();   // every warp is done with the previous chunk's rows
            // h of (expert d0 + r / 4, its (r % 4)-th token) into row r
            stage_rows(smem, 4 * min(cpe, 2), p.k, [&](int r) -> const float* {
                const int dd = d0 + r / 4, j = r % 4;
                if (dd >= nd) return nullptr;
                const unsigned m = (unsigned)s_mask[dd];
                if (j >= __popc(m)) return nullptr;
                const int t = nth_bit(m, j);   // the expert's j-th token
                return p.h + (size_t)s_first[dd * kMaxTok + t] * p.ff;
            });
        }
        first_chunk = false;
        for (int m = pos; pos < P && m < ce - cs; m += P) {
            const int sq = seq + m;
            const int s = sq % kStages;
            const bool stamped = wait_seq(&descs[s].seq, sq, p.err, abort_flag);
            const bool landed = stamped && mbar_wait(full0 + 8 * s, (sq / kStages) & 1, p.err, abort_flag);
            // without a stamp the descriptor is not this item's: it is not used
            const int dd = stamped ? descs[s].d : d0, r = stamped ? descs[s].r : 0;
            const int bad = !stamped ? -1 : !landed ? SB_DERR_TIMEOUT : descs[s].bad;
            // this lane's B column g: GU token g / 2, down the expert's (g / 2)-th token; part g % 2
            const int brow = GU ? (g >> 1) : 4 * (dd - d0) + (g >> 1);
            const bool have = GU ? (g >> 1) < p.n_tokens : (g >> 1) < __popc((unsigned)s_mask[dd]);
            const uint32_t bcol = smem_u32(smem + Smem::barea) + (uint32_t)(brow * stride + ((g & 1) ? kLoOff : 0));
            const int crow = (GU ? c : 4 * (dd - d0) + c) * gpr;   // column c's staged row
            float acc[2] = {0.f, 0.f};
            if (!bad) {
                const uint32_t tile = smem_u32(smem + Smem::stages) + (uint32_t)(s * kStageBytes);
                KQ<QT>::superblock(tile, p.rs, wsub, g, c, bcol, have, smem_u32(sums + crow), smem_u32(invs + crow), acc);
            }
            red[(s * kMaxWpt + wsub) * 32 + lane] = make_float2(acc[0], acc[1]);
            __threadfence_block();
            __syncwarp();
            int last = 0;
            if (lane == 0) {
                last = atomicAdd(cnt + s, 1) == wpt - 1;
                if (last) cnt[s] = 0;
            }
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            // ---- epilogue (the item's last warp): the warps' partial rows in fixed order
            __threadfence_block();
            float v0 = 0.f, v1 = 0.f;
            for (int w = 0; w < wpt; ++w) {
                const float2 q = red[(s * kMaxWpt + w) * 32 + lane];
                v0 += q.x;
                v1 += q.y;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * s);   // the stage and its red slot may be reused
            if (bad < 0) continue;   // aborting: the error is recorded
            if (bad > 0) {
                v0 = v1 = __int_as_float(0x7fc00000);
                if (lane == 0 && p.err) atomicExch(p.err, bad);
            }
            // every pair routed to expert dd; lanes of column c hold its token
            const unsigned m0 = __ballot_sync(0xffffffffu, lane < n_pairs && s_dist[lane] == dd);
            const unsigned m1 = __ballot_sync(0xffffffffu, lane + 32 < n_pairs && s_dist[lane + 32] == dd);
            const unsigned mask = (unsigned)s_mask[dd];
            if (GU) {
                // column c is token c: rows g (gate) and g + 8 (up) of 8-row block r
                const float gv = v0, uv = v1;
                const float hv = gv / (1.f + expf(-gv)) * uv;
                for (int half = 0; half < 2; ++half)
                    for (unsigned mm = half ? m1 : m0; mm; mm &= mm - 1) {
                        const int pr = __ffs(mm) - 1 + 32 * half;
                        if (pr / p.n_used == c) p.h[(size_t)pr * p.ff + 8 * r + g] = hv;
                    }
            } else {
                // column c is the expert's c-th token: rows g and g + 8 of 16-row tile r
                if (c < __popc(mask)) {
                    const int t = nth_bit(mask, c);
                    for (int half = 0; half < 2; ++half)
                        for (unsigned mm = half ? m1 : m0; mm; mm &= mm - 1) {
                            const int pr = __ffs(mm) - 1 + 32 * half;
                            if (pr / p.n_used == t) {
                                float* o = p.v + (size_t)pr * p.d_model + 16 * r;
                                o[g] = v0;
                                o[g + 8] = v1;
                            }
                        }
                }
            }
        }
        seq += ce - cs;
    }
}

// out[t][i] = (accumulate ? out[t][i] : 0) + sum_e w[t][e] * v[t][e][i], slots
// in order (k_down's order); a pair with a bad id contributes NaN. The
// weights (NaN for bad ids) are read once per CTA into shared memory.
__global__ void k_small_combine(const SmallParams p, const float* w, float* out, int accumulate) {
    __shared__ float s_w[kMaxPairs];
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int n_pairs = p.n_tokens * p.n_used;
    for (int q = threadIdx.x; q < n_pairs; q += blockDim.x) {
        const int t = q / p.n_used, e = q % p.n_used;
        const int id = *(const int32_t*)(p.ids + (size_t)t * p.ids_token_stride + (size_t)e * p.ids_id_stride);
        s_w[q] = (id < 0 || id >= p.n_experts) ? __int_as_float(0x7fc00000) : w[q];
    }
    __syncthreads();
    const long long n = (long long)p.n_tokens * p.d_model;
    for (long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x; q < n; q += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(q / p.d_model), i = (int)(q % p.d_model);
        const float* vr = p.v + (size_t)t * p.n_used * p.d_model + i;
        const float* wr = s_w + t * p.n_used;
        float tot = 0.f;
        int e = 0;
        for (; e + 4 <= p.n_used; e += 4) {
            const float y0 = __ldcg(vr + (size_t)e * p.d_model), y1 = __ldcg(vr + (size_t)(e + 1) * p.d_model);
            const float y2 = __ldcg(vr + (size_t)(e + 2) * p.d_model), y3 = __ldcg(vr + (size_t)(e + 3) * p.d_model);
            // a NaN weight marks a bad id: its product is NaN whatever v holds
            tot += wr[e] != wr[e] ? wr[e] : wr[e] * y0;
            tot += wr[e + 1] != wr[e + 1] ? wr[e + 1] : wr[e + 1] * y1;
            tot += wr[e + 2] != wr[e + 2] ? wr[e + 2] : wr[e + 2] * y2;
            tot += wr[e + 3] != wr[e + 3] ? wr[e + 3] : wr[e + 3] * y3;
        }
        for (; e < p.n_used; ++e) {
            const float y = __ldcg(vr + (size_t)e * p.d_model);
            tot += wr[e] != wr[e] ? wr[e] : wr[e] * y;
        }
        out[q] = accumulate ? out[q] + tot : tot;
    }
}

// ------------------------------------------------------------ host side
struct SmallScratch {
    float* v = nullptr;
    size_t cap = 0;   // floats
};
SmallScratch g_ss;
int g_sms = 0;
bool g_attr[4] = {false, false, false, false};

// SABAH_KQ_PAD=0 copies tiles whole even where rows would share banks
bool pad_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* v = std::getenv("SABAH_KQ_PAD");
        on = !(v && *v == '0');
    }
    return on != 0;
}

bool small_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* v = std::getenv("SABAH_KQ_SMALL");
        on = !(v && *v == '0');
    }
    return on != 0;
}

// staged row stride: the 8 rows an MMA reads at one offset fall into 8
// different 16-byte bank groups when the stride is an odd number of 16-byte
// units; rows that are an even number of units get 16 bytes of padding (and
// row-by-row copies)
int staged_stride(int rb) { return (pad_enabled() && rb % 16 == 0 && (rb / 16) % 2 == 0) ? rb + 16 : rb; }

// launched with programmatic stream serialization (see the kernel)
template <class K, class... Args>
bool launch_pdl(K kernel, int grid, int threads, int smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return sb_cuda_ok(cudaLaunchKernelEx(&cfg, kernel, args...), "small-batch launch");
}

template <int QT, bool GU>
bool launch_small(const SmallParams& p, cudaStream_t st, int slot) {
    if (!g_attr[slot]) {
        if (!sb_cuda_ok(cudaFuncSetAttribute(k_small<QT, GU>, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::total),
                        "small-batch smem attribute"))
            return false;
        g_attr[slot] = true;
    }
    return launch_pdl(k_small<QT, GU>, g_sms, kThreads, Smem::total, st, p);
}

bool kq_type(int qt) { return qt == SB_Q4_K || qt == SB_Q6_K; }

}  // namespace

int sb_try_block_small(const sb_block_args& a, cudaStream_t st) {
    if (!small_enabled() || a.qt_gate != a.qt_up || !kq_type(a.qt_gate) || !kq_type(a.qt_down)) return 0;
    if (a.gate.ptrs || a.up.ptrs || a.down.ptrs || !a.gate.base || !a.up.base || !a.down.base || !a.gate.ids) return 0;
    if (a.n_tokens < 1 || a.n_tokens > kMaxTok || a.n_used < 1 || a.n_tokens * a.n_used > kMaxPairs) return 0;
    if (a.d_model % 256 || a.ff % 256 || a.d_model > 2048 || a.ff > 2048) return 0;
    const int rb_gu = (int)sb_row_bytes_of(a.qt_gate, a.d_model), rb_dn = (int)sb_row_bytes_of(a.qt_down, a.ff);
    const int rs_gu = staged_stride(rb_gu), rs_dn = staged_stride(rb_dn);
    if (16 * rs_gu > kStageBytes || 16 * rs_dn > kStageBytes || (8 * rb_gu) % 16 || (16 * rb_dn) % 16) return 0;
    for (const sb_experts* e : {&a.gate, &a.up, &a.down})
        if (((uintptr_t)e->base & 15) || e->expert_stride % 16 || e->n_experts < 1) return 0;
    if (a.gate.ids != a.up.ids || a.gate.ids != a.down.ids) return 0;
    if (((uintptr_t)a.x & 15) || ((uintptr_t)a.h & 15) || !a.out || !a.w) return 0;

    const size_t need = (size_t)a.n_tokens * a.n_used * a.d_model;
    if (need > g_ss.cap) {
        if (g_ss.v) {
            cudaDeviceSynchronize();   // no kernel of an earlier call may still use it
            cudaFree(g_ss.v);
        }
        g_ss = SmallScratch{};
        if (!sb_cuda_ok(cudaMalloc(&g_ss.v, need * sizeof(float)), "small-batch scratch")) return -1;
        g_ss.cap = need;
    }
    if (!g_sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_sms < 1) g_sms = 148;
    }
    SmallParams p{};
    p.gate = a.gate.base;
    p.up = a.up.base;
    p.down = a.down.base;
    p.gu_stride = a.gate.expert_stride;
    p.dn_stride = a.down.expert_stride;
    p.ids = (const uint8_t*)a.gate.ids;
    p.ids_id_stride = a.gate.ids_id_stride;
    p.ids_token_stride = a.gate.ids_token_stride;
    p.n_experts = a.gate.n_experts;
    p.n_tokens = a.n_tokens;
    p.n_used = a.n_used;
    p.d_model = a.d_model;
    p.ff = a.ff;
    p.x = a.x;
    p.h = a.h;
    p.v = g_ss.v;
    p.err = a.err;

    const int t1 = sb_timing_begin("small_kq_gate_up", st);
    SmallParams pg = p;
    pg.rb = rb_gu;
    pg.rs = rs_gu;
    pg.k = a.d_model;
    pg.rows_out = a.ff;
    const bool ok1 = a.qt_gate == SB_Q4_K ? launch_small<SB_Q4_K, true>(pg, st, 0) : launch_small<SB_Q6_K, true>(pg, st, 1);
    sb_timing_end(t1, st);
    if (!ok1) return -1;
    const int t2 = sb_timing_begin("small_kq_down", st);
    SmallParams pd = p;
    pd.ids_ready = 1;   // launched right after this call's gate/up kernel
    pd.rb = rb_dn;
    pd.rs = rs_dn;
    pd.k = a.ff;
    pd.rows_out = a.d_model;
    const bool ok2 = a.qt_down == SB_Q4_K ? launch_small<SB_Q4_K, false>(pd, st, 2) : launch_small<SB_Q6_K, false>(pd, st, 3);
    sb_timing_end(t2, st);
    if (!ok2) return -1;
    const int t3 = sb_timing_begin("small_kq_combine", st);
    const long long n = (long long)a.n_tokens * a.d_model;
    const bool ok3 = launch_pdl(k_small_combine, (int)std::min<long long>((n + 255) / 256, 4LL * g_sms), 256, 0, st, pd,
                                a.w, a.out, a.accumulate);
    sb_timing_end(t3, st);
    return ok3 ? 1 : -1;
}
