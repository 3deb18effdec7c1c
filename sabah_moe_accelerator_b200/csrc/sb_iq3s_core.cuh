// Decode core of the IQ3_S kernels (sb_mmid_iq3s.cu: one launch per matrix or
// block; sb_decode_iq3s.cu: one persistent launch per token): PTX helpers, the
// x-fragment sets and the tensor-core decode of a super-block pair. The
// technique is described at the top of sb_mmid_iq3s.cu.
#pragma once

#include <cuda_fp16.h>

#include <utility>

#include "sb_kernels.h"
#include "sb_quant.cuh"

namespace sb_iq3s {

// Grid-table replicas: lane l reads replica l % R, so a warp's 32 lookups meet
// at most 32 / R entries per bank word column (R = 16: 32 KB; R = 32: 64 KB,
// conflict-free).
constexpr int kReplicas = 16;
constexpr int kTableBytes = 512 * kReplicas * 4; // 32 KB
template <int R>
constexpr int table_bytes() { return 512 * R * 4; }
// A producer lane issues its bulk copies one after another (~0.34 us apiece),
// so kIssuers lanes share the issuing; each owns every kIssuers-th stage.
constexpr int kIssuers = 8;
constexpr int kRecBytes = 72;                    // per (group, step): 4 quads x (hi, lo) x 8 B + 8 B zeros
constexpr int kGroupBytes = 8 * kRecBytes + 16;  // 8 records + 4 per-sub-block inverse scales
constexpr int kSetBytes = 16 * kGroupBytes;      // k <= 2048
constexpr int kSuspendNs = 20000;                // try_wait suspend hint
constexpr long long kSpinLimit = 1ll << 17;      // bounded waits: <= 2^17 x 20 us ~ 2.6 s

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
// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps (up to the hint) instead of spinning, so waiting producer lanes and
// consumers do not steal issue slots from the warps that are decoding
template <int HINT_NS = kSuspendNs>
__device__ inline bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "n"(HINT_NS)
        : "memory");
    return ok != 0;
}
// Bounded wait. False when the CTA is aborting or when this wait gives up (it
// then sets the abort flag and the device error word). Callers skip their work
// but keep taking part in every barrier, so nothing is left waiting.
template <int HINT_NS = kSuspendNs>
__device__ inline bool mbar_wait(uint32_t bar, uint32_t parity, int* err, volatile int* abort_flag) {
    const long long limit = kSpinLimit * (kSuspendNs / HINT_NS);   // the same ~2.6 s bound for any hint
    for (long long i = 0; i < limit; ++i) {
        if (mbar_try_wait<HINT_NS>(bar, parity)) return true;
        if ((i & 15) == 15 && *abort_flag) return false;
    }
    *abort_flag = 1;
    if (err) atomicExch(err, SB_DERR_TIMEOUT);
    return false;
}
// Bounded wait for the producer's sequence stamp on a stage descriptor.
__device__ inline bool wait_seq(const int* stamp, int seq, int* err, volatile int* abort_flag) {
    const volatile int* v = stamp;
    for (long long i = 0; i < kSpinLimit * 64; ++i) {
        if (*v == seq) return true;
        if (*abort_flag) return false;
        __nanosleep(64);
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

// shared-memory loads at 32-bit addresses with a compile-time offset (keeps the
// address arithmetic out of the decode loop)
template <int OFF>
__device__ inline uint32_t ld_u8(uint32_t a) {
    uint32_t v;
    asm("ld.shared.u8 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF));
    return v;
}
template <int OFF>
__device__ inline uint32_t ld_u16(uint32_t a) {
    uint32_t v;
    asm("ld.shared.u16 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF));
    return v;
}
template <int OFF>
__device__ inline uint32_t ld_u32(uint32_t a) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(a), "n"(OFF));
    return v;
}
template <int OFF>
__device__ inline uint2 ld_v2(uint32_t a) {
    uint2 v;
    asm("ld.shared.v2.u32 {%0,%1}, [%2+%3];" : "=r"(v.x), "=r"(v.y) : "r"(a), "n"(OFF));
    return v;
}
template <int OFF>
__device__ inline float ld_f32(uint32_t a) {
    float v;
    asm("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(a), "n"(OFF));
    return v;
}

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

// ---------------------------------------------------------------- x fragments
// B-operand set of vector x (length k): group q holds records (q, step s) with,
// for quad c, hi and lo half2 pairs of elements 32*(4q+c) + 4s .. +3 (scaled
// per sub-block), a zero pair, then the 4 inverse scales of its sub-blocks.
// Float4 f of x = entry f % 8 of sub-block f / 8. Threads 0..NT-1 build; NT is
// a multiple of 32 and whole warps take part (the max uses warp shuffles).
// x-fragments of float4 f of one vector (v4) into set `set`; lanes of a warp
// hold 32 consecutive float4 of the same vector.
__device__ inline void set_put(float4 v4, int f, uint8_t* set) {
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

// build_sets_from builds the sets of n_keys vectors in one pass: float4 f of
// vector i comes from load(i, f) (so x can be formed on the fly) and goes to
// set set_of(i). k is a multiple of 128, so a warp never straddles two
// vectors. kLoadRounds rounds of loads are issued before any is used.
template <int NT, class Load, class SetOf, int kLoadRounds = 2>
__device__ inline void build_sets_from(int n_keys, Load load, SetOf set_of, int k) {
    const int nf = k / 4, total = n_keys * nf;
    for (int base = 0; base < total; base += kLoadRounds * NT) {
        float4 v[kLoadRounds];
#pragma unroll
        for (int u = 0; u < kLoadRounds; ++u) {
            const int idx = base + u * NT + (int)threadIdx.x;
            if (idx < total) v[u] = load(idx / nf, idx % nf);
        }
#pragma unroll
        for (int u = 0; u < kLoadRounds; ++u) {
            const int idx = base + u * NT + (int)threadIdx.x;
            if (idx < total) set_put(v[u], idx % nf, set_of(idx / nf));
        }
    }
}

template <int NT>
__device__ inline void build_set(const float* x, int k, uint8_t* set) {
    build_sets_from<NT>(
        1, [x](int, int f) { return __ldcg((const float4*)x + f); }, [set](int) { return set; }, k);
}

// ---------------------------------------------------------------- decode core
// Per-thread constant addresses (32-bit shared-memory addresses).
struct Lane {
    uint32_t table;    // replica (lane % 16) of the grid table
    uint32_t invd;     // from a lane's B record to its quad's inverse scale: 4c - boff (mod 2^32)
    uint32_t row8c;    // tile-relative offsets of row g: + 8c (qs), + 4c (signs), + c (qh), + c/2 (scales)
    uint32_t row4c, row1c, rowhc, row0;
    uint32_t rb8;      // 8 rows
    int nib_shift;     // 4 * (c & 1): the scale nibble of sub-block 4n + c
};

// Per-(row, sub-block) fields of group N of a pair (N = 0: sub-block c of the
// super-block, N = 1: sub-block 4 + c): the 8 qs bytes (4 u16), the 4 sign
// bytes, the qh byte spread to one 0/1 byte per entry (the 9th index bit), and
// the sub-block scale db = d * (1 + 2 * nibble) * (x inverse scale).
template <int N>
__device__ inline void load_fields(uint32_t r8, uint32_t r4, uint32_t r1, uint32_t rh, uint32_t invq, int nib_shift,
                                   float d, uint32_t (&qsw)[4], uint32_t (&QH)[2], uint32_t (&sgw)[4], float& db) {
    qsw[0] = ld_u16<2 + 32 * N>(r8);
    qsw[1] = ld_u16<4 + 32 * N>(r8);
    qsw[2] = ld_u16<6 + 32 * N>(r8);
    qsw[3] = ld_u16<8 + 32 * N>(r8);
    sgw[0] = ld_u8<74 + 16 * N>(r4);
    sgw[1] = ld_u8<75 + 16 * N>(r4);
    sgw[2] = ld_u8<76 + 16 * N>(r4);
    sgw[3] = ld_u8<77 + 16 * N>(r4);
    const uint32_t qh = ld_u8<66 + 4 * N>(r1);
    QH[0] = ((qh & 15u) * 0x00204081u) & 0x01010101u;   // qh bits 0..3 -> bytes 0..3
    QH[1] = ((qh >> 4) * 0x00204081u) & 0x01010101u;    // qh bits 4..7 -> bytes 0..3
    const uint32_t nib = (ld_u8<106 + 2 * N>(rh) >> nib_shift) & 15u;
    const float inv = ld_f32<N * kGroupBytes + 8 * kRecBytes>(invq);
    db = d * (float)(1 + 2 * (int)nib) * inv;
}

// Step S (grid entry S of every sub-block) of both groups of a pair: decode
// rows g and g + 8 of entry S into A fragments and issue the two MMAs.
template <int S, int LOG_R>
__device__ inline void step(uint32_t setq, uint32_t table, const uint32_t (&qsw)[2][2][4], const uint32_t (&QH)[2][2][2],
                            const uint32_t (&sgw)[2][2][4], float (&dd)[2][4]) {
    // PRMT selector: byte 0 = qs byte (S & 1) of the u16 word, byte 1 = QH byte (S & 3), bytes 2, 3 = 0
    constexpr uint32_t sel = (uint32_t)(S & 1) | ((4u + (S & 3)) << 4) | (2u << 8) | (2u << 12);
    constexpr uint32_t mask = (S & 1) ? 0xF0u : 0x0Fu;                 // entry S's sign nibble
    constexpr uint32_t kspread = (S & 1) ? 0x01020408u : 0x10204080u;  // nibble bits -> bit 7 of bytes 0..3
    const uint2 bv[2] = {ld_v2<S * kRecBytes>(setq), ld_v2<kGroupBytes + S * kRecBytes>(setq)};
#pragma unroll
    for (int n = 0; n < 2; ++n) {
        uint32_t a[2][2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t idx = prmt(qsw[n][h][S >> 1], QH[n][h][S >> 2], sel);
            uint32_t grid;
            asm("ld.shared.u32 %0, [%1];" : "=r"(grid) : "r"((idx << (LOG_R + 2)) + table));
            const uint32_t Z = ((sgw[n][h][S >> 1] & mask) * kspread) & 0x80808080u;
            a[h][0] = prmt(grid, Z, 0x5140);   // (e0, e1) as signed fp16 subnormals
            a[h][1] = prmt(grid, Z, 0x7362);   // (e2, e3)
        }
        mma16816(dd[n], a[0][0], a[1][0], a[0][1], a[1][1], bv[n].x, bv[n].y);
    }
}

template <int LOG_R, int... S>
__device__ inline void all_steps(std::integer_sequence<int, S...>, uint32_t setq, uint32_t table,
                                 const uint32_t (&qsw)[2][2][4], const uint32_t (&QH)[2][2][2],
                                 const uint32_t (&sgw)[2][2][4], float (&dd)[2][4]) {
    (step<S, LOG_R>(setq, table, qsw, QH, sgw, dd), ...);
}

// Decode the group pair (q, q + 1), q even (the two halves of super-block q / 2),
// of a 16-row tile at shared address tile: 2 interleaved MMA chains; adds the
// sub-block dots of rows g and g + 8 into acc[0] and acc[1]. setB = x-set base
// + this lane's B-record offset.
template <int LOG_R = 4>
__device__ inline void do_pair(uint32_t tile, int q, uint32_t setB, const Lane& L, float (&acc)[2]) {
    const uint32_t sb = tile + (uint32_t)(q >> 1) * 110u;
    const uint32_t setq = setB + (uint32_t)q * kGroupBytes;
    const uint32_t invq = setq + L.invd;
    uint32_t qsw[2][2][4], QH[2][2][2], sgw[2][2][4];
    float db[2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t r8 = sb + L.row8c + h * L.rb8, r4 = sb + L.row4c + h * L.rb8;
        const uint32_t r1 = sb + L.row1c + h * L.rb8, rh = sb + L.rowhc + h * L.rb8;
        const float d = __half2float(__ushort_as_half((unsigned short)ld_u16<0>(sb + L.row0 + h * L.rb8)));
        load_fields<0>(r8, r4, r1, rh, invq, L.nib_shift, d, qsw[0][h], QH[0][h], sgw[0][h], db[0][h]);
        load_fields<1>(r8, r4, r1, rh, invq, L.nib_shift, d, qsw[1][h], QH[1][h], sgw[1][h], db[1][h]);
    }
    float dd[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) dd[n][0] = dd[n][1] = dd[n][2] = dd[n][3] = 0.f;
    all_steps<LOG_R>(std::make_integer_sequence<int, 8>{}, setq, L.table, qsw, QH, sgw, dd);
#pragma unroll
    for (int n = 0; n < 2; ++n) {
        acc[0] = fmaf(db[n][0], dd[n][0] + dd[n][1], acc[0]);
        acc[1] = fmaf(db[n][1], dd[n][2] + dd[n][3], acc[1]);
    }
}

// ---------------------------------------------------------------- Q8_0 decode
// The same engine for Q8_0 (34-byte blocks of 32 weights: fp16 d, then 32
// int8): a block is a sub-block of the K permutation (quad c owns block
// 4q + c of group q), so the x sets and MMA chains are those of IQ3_S. In
// shared memory a tile's rows come in pairs (2g, 2g + 1), one bulk copy each,
// at a padded pair stride, so a warp's loads of rows 2g (g = 0..7) spread over
// the banks; lane (g, c) decodes rows 2g (h = 0) and 2g + 1 (h = 1).
struct LaneQ8 {
    uint32_t row;     // tile-relative offset of row 2g (row 2g + 1 is rb further)
    uint32_t rb;
    uint32_t qoff;    // 34c + 2 rounded down to 4: block c's first aligned quant word
    uint32_t dof;     // 34c: block c's scale
    uint32_t sel;     // PRMT selector for 4 quants from words (j, j + 1)
    uint32_t invd;    // as Lane::invd
};
__device__ inline LaneQ8 lane_init_q8(int rb, int pair_stride, int lane) {
    const int g = lane >> 2, c = lane & 3;
    const int boff = (g >> 1) == c ? (2 * c + (g & 1)) * 8 : 64;
    LaneQ8 L;
    L.row = (uint32_t)(g * pair_stride);
    L.rb = (uint32_t)rb;
    L.dof = (uint32_t)(34 * c);
    L.qoff = (uint32_t)((34 * c + 2) & ~3);
    L.sel = (c & 1) ? 0x3210u : 0x5432u;   // c odd: block c's quants are word-aligned
    L.invd = (uint32_t)(4 * c - boff);
    return L;
}

__device__ inline uint32_t hsub2_u32(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// Weights 4S .. 4S + 3 of a block (words w0, w1 around them) as two fp16
// pairs: biased bytes b = q + 128 placed under exponent 0x64 give 1024 + b
// exactly; subtracting 1152 leaves q.
__device__ inline void q8_entry(uint32_t w0, uint32_t w1, uint32_t sel, uint32_t& a0, uint32_t& a1) {
    const uint32_t u = prmt(w0, w1, sel) ^ 0x80808080u;
    a0 = hsub2_u32(prmt(u, 0x64646464u, 0x4140u), 0x64806480u);
    a1 = hsub2_u32(prmt(u, 0x64646464u, 0x4342u), 0x64806480u);
}

// Step S (weights 4S .. 4S + 3 of every block) of both groups of a Q8_0 pair;
// w holds word S of each (group, row) and advances to word S + 1.
template <int S>
__device__ inline void step_q8(uint32_t setq, uint32_t sel, const uint32_t (&base)[2][2], uint32_t (&w)[2][2],
                               float (&dd)[2][4]) {
    const uint2 bv[2] = {ld_v2<S * kRecBytes>(setq), ld_v2<kGroupBytes + S * kRecBytes>(setq)};
#pragma unroll
    for (int n = 0; n < 2; ++n) {
        uint32_t a[2][2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t wn = ld_u32<4 * (S + 1)>(base[n][h]);
            q8_entry(w[n][h], wn, sel, a[h][0], a[h][1]);
            w[n][h] = wn;
        }
        mma16816(dd[n], a[0][0], a[1][0], a[0][1], a[1][1], bv[n].x, bv[n].y);
    }
}
template <int... S>
__device__ inline void all_steps_q8(std::integer_sequence<int, S...>, uint32_t setq, uint32_t sel,
                                    const uint32_t (&base)[2][2], uint32_t (&w)[2][2], float (&dd)[2][4]) {
    (step_q8<S>(setq, sel, base, w, dd), ...);
}

// Group pair (q, q + 1) of a Q8_0 tile: blocks 4q + c and 4q + 4 + c of rows
// 2g and 2g + 1; adds their dots into acc[0] (row 2g) and acc[1] (row 2g + 1).
__device__ inline void do_pair_q8(uint32_t tile, int q, uint32_t setB, const LaneQ8& L, float (&acc)[2]) {
    const uint32_t setq = setB + (uint32_t)q * kGroupBytes;
    const uint32_t invq = setq + L.invd;
    uint32_t base[2][2], w[2][2];
    float db[2][2];
#pragma unroll
    for (int n = 0; n < 2; ++n) {
        // the set's inverse scale carries 2^24 for IQ3_S's subnormal weights; Q8_0 quants are plain fp16
        const float inv = ld_f32<8 * kRecBytes>(invq + (uint32_t)n * kGroupBytes) * (1.0f / 16777216.0f);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t blk = tile + L.row + (uint32_t)h * L.rb + (uint32_t)(q + n) * 136u;
            base[n][h] = blk + L.qoff;
            w[n][h] = ld_u32<0>(base[n][h]);
            db[n][h] = __half2float(__ushort_as_half((unsigned short)ld_u16<0>(blk + L.dof))) * inv;
        }
    }
    float dd[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) dd[n][0] = dd[n][1] = dd[n][2] = dd[n][3] = 0.f;
    all_steps_q8(std::make_integer_sequence<int, 8>{}, setq, L.sel, base, w, dd);
#pragma unroll
    for (int n = 0; n < 2; ++n) {
        acc[0] = fmaf(db[n][0], dd[n][0] + dd[n][1], acc[0]);
        acc[1] = fmaf(db[n][1], dd[n][2] + dd[n][3], acc[1]);
    }
}

// Replicated grid table: entry e, replica r at word e * kReplicas + r. Threads
// 0..NT-1 fill it.
template <int NT, int R = kReplicas>
__device__ inline void fill_table(uint32_t* table) {
    for (int e = threadIdx.x; e < 512; e += NT) {
        const uint32_t w = sb_iq3s_grid[e];
        uint4* dst = (uint4*)(table + e * R);
#pragma unroll
        for (int r = 0; r < R / 4; ++r) dst[r] = make_uint4(w, w, w, w);
    }
}

// This lane's constant addresses for tiles with rows of rb bytes.
template <int R = kReplicas>
__device__ inline Lane lane_init(const uint32_t* table, int rb, int lane) {
    const int g = lane >> 2, c = lane & 3;
    const int boff = (g >> 1) == c ? (2 * c + (g & 1)) * 8 : 64;
    Lane L;
    L.table = smem_u32(table) + (lane & (R - 1)) * 4;
    L.invd = (uint32_t)(4 * c - boff);
    L.row0 = (uint32_t)(g * rb);
    L.row8c = L.row0 + 8 * c;
    L.row4c = L.row0 + 4 * c;
    L.row1c = L.row0 + c;
    L.rowhc = L.row0 + (c >> 1);
    L.rb8 = (uint32_t)(8 * rb);
    L.nib_shift = 4 * (c & 1);
    return L;
}
// Offset of this lane's B record inside a group (the x-set base is added).
__device__ inline uint32_t lane_boff(int lane) {
    const int g = lane >> 2, c = lane & 3;
    return (uint32_t)((g >> 1) == c ? (2 * c + (g & 1)) * 8 : 64);
}

}  // namespace sb_iq3s
