// Decode core of the barrier-free one-token kernel (sb_flow_iq3s.cu): B
// fragments built in registers from 128 values of a vector, and the decode of
// one 128-weight group of a 16-row IQ3_S tile (or of two tiles at once) on
// mma.sync, over the helpers of sb_iq3s_core.cuh.
#pragma once

#include "sb_iq3s_core.cuh"

namespace sb_flow {

using namespace sb_iq3s;

// Grid-table format (1 measured about 10% faster on B200 in the decode core
// alone). 0: 4-byte entries (the grid bytes), 32 replicas, signs
// placed by a multiply-spread and two PRMTs. 1: 8-byte entries holding the
// entry already as two fp16-subnormal pairs, 16 replicas (a half-warp's
// 8-byte loads hit distinct bank pairs), signs applied by two IMAD + LOP3.
// Both tables are 64 KB: 128 bytes per entry across the replicas.
#ifndef SB_FLOW_TABLE64
#define SB_FLOW_TABLE64 1
#endif
constexpr bool kTable64 = SB_FLOW_TABLE64 != 0;
constexpr int kR = kTable64 ? 16 : 32;
constexpr int kGridBytes = 512 * 128;

template <int NT>
__device__ inline void fill_grid(uint32_t* table) {
    for (int e = threadIdx.x; e < 512; e += NT) {
        const uint32_t w = sb_iq3s_grid[e];
        if (kTable64) {
            const uint32_t lo = (w & 0xFFu) | ((w & 0xFF00u) << 8), hi = ((w >> 16) & 0xFFu) | ((w >> 8) & 0xFF0000u);
            uint4* dst = (uint4*)(table + e * 32);
#pragma unroll
            for (int r = 0; r < 8; ++r) dst[r] = make_uint4(lo, hi, lo, hi);
        } else {
            uint4* dst = (uint4*)(table + e * 32);
#pragma unroll
            for (int r = 0; r < 8; ++r) dst[r] = make_uint4(w, w, w, w);
        }
    }
}
// this lane's replica of the grid table
__device__ inline uint32_t grid_lane(const uint32_t* table, int lane) {
    return smem_u32(table) + (kTable64 ? (uint32_t)(lane & 15) * 8u : (uint32_t)(lane & 31) * 4u);
}

// Entry S of a (row, sub-block): the 9-bit grid index from the qs word and the
// spread qh word, the grid value and the entry's 4 sign bits from the sign
// byte -> A fragments (e0, e1), (e2, e3) as signed fp16 subnormals.
template <int S>
__device__ inline void decode_entry(uint32_t qs, uint32_t qh, uint32_t sbyte, uint32_t tab, uint32_t& a0,
                                    uint32_t& a1) {
    // PRMT selector: byte 0 = qs byte (S & 1) of the u16 word, byte 1 = QH byte (S & 3), bytes 2, 3 = 0
    constexpr uint32_t sel = (uint32_t)(S & 1) | ((4u + (S & 3)) << 4) | (2u << 8) | (2u << 12);
    const uint32_t idx = prmt(qs, qh, sel);
    if (kTable64) {
        uint32_t g0, g1;
        asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(g0), "=r"(g1) : "r"((idx << 7) + tab));
        // sign bits (4S .. 4S + 3 of the byte pair) to bits 15 and 31 of each pair
        constexpr uint32_t k0 = (S & 1) ? 0x04000800u : 0x40008000u;
        constexpr uint32_t k1 = (S & 1) ? 0x01000200u : 0x10002000u;
        a0 = g0 ^ ((sbyte * k0) & 0x80008000u);
        a1 = g1 ^ ((sbyte * k1) & 0x80008000u);
    } else {
        constexpr uint32_t mask = (S & 1) ? 0xF0u : 0x0Fu;                 // entry S's sign nibble
        constexpr uint32_t kspread = (S & 1) ? 0x01020408u : 0x10204080u;  // nibble bits -> bit 7 of bytes 0..3
        uint32_t grid;
        asm("ld.shared.u32 %0, [%1];" : "=r"(grid) : "r"((idx << 7) + tab));
        const uint32_t Z = ((sbyte & mask) * kspread) & 0x80808080u;
        a0 = prmt(grid, Z, 0x5140);
        a1 = prmt(grid, Z, 0x7362);
    }
}

// B operand of mma.sync m16n8k16 for one 128-element group of a vector, lane
// l holding elements [4l, 4l + 4). One power-of-two scale for the group puts
// its max into [2^13, 2^14) (a warp max reduction, REDUX); each value splits
// into fp16 hi and lo parts, which keep about 22 bits of it. stage_b writes
// lane l's (hi01, hi23, lo01, lo23) to the warp's 512-byte staging area and
// returns 2^24 / scale (the 2^24 undoes the subnormal encoding of the weights).
__device__ inline float stage_b(float4 v4, uint32_t bst) {
    const int lane = threadIdx.x & 31;
    const float m = fmaxf(fmaxf(fabsf(v4.x), fabsf(v4.y)), fmaxf(fabsf(v4.z), fabsf(v4.w)));
    // positive floats order as their bit patterns; NaN and inf give no scaling
    const unsigned mb = __reduce_max_sync(0xffffffffu, __float_as_uint(m));
    const int E = (int)(mb >> 23);   // biased exponent of the max: max = f * 2^(E - 126), f in [0.5, 1)
    const int ex = (mb == 0u || E == 255) ? 0 : max(-100, min(100, 14 - (E - 126)));
    const float s = __int_as_float((ex + 127) << 23);
    const float2 a = make_float2(v4.x * s, v4.y * s), b = make_float2(v4.z * s, v4.w * s);
    const __half2 h01 = __float22half2_rn(a), h23 = __float22half2_rn(b);
    const float2 ra = __half22float2(h01), rb = __half22float2(h23);
    const __half2 l01 = __float22half2_rn(make_float2(a.x - ra.x, a.y - ra.y));
    const __half2 l23 = __float22half2_rn(make_float2(b.x - rb.x, b.y - rb.y));
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(bst + 16u * lane), "r"(*(const uint32_t*)&h01),
                 "r"(*(const uint32_t*)&h23), "r"(*(const uint32_t*)&l01), "r"(*(const uint32_t*)&l23)
                 : "memory");
    return __int_as_float((24 - ex + 127) << 23);
}

// Lane (g, c)'s B fragment of step S from a staged group: the hi (g even) or
// lo (g odd) pairs of entry S of sub-block c when g / 2 == c, zeros otherwise
// (the K permutation of the decode core).
__device__ inline void load_b(uint32_t bst, int S, uint32_t& b0, uint32_t& b1) {
    const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    b0 = b1 = 0;
    if ((g >> 1) == c)
        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(b0), "=r"(b1)
                     : "r"(bst + 16u * (8 * c + S) + 8u * (g & 1)));
}

// B fragments of all 8 steps in registers (the gate/up path keeps them for
// every item of a layer).
__device__ inline void build_b(float4 v4, uint32_t bst, uint32_t (&bf)[8][2], float& inv) {
    inv = stage_b(v4, bst);
    __syncwarp();
#pragma unroll
    for (int S = 0; S < 8; ++S) load_b(bst, S, bf[S][0], bf[S][1]);
    __syncwarp();   // the staging area may be rewritten after this
}

// Fields of rows g (h = 0) and g + 8 (h = 1) for sub-block 4N + c of the
// super-block at shared address sb (row 0): 8 qs bytes (4 u16), 4 sign
// bytes, the qh byte spread to one 0/1 byte per entry, and the scale
// db = d * (1 + 2 * nibble) * inv.
template <int N>
__device__ inline void fields(uint32_t sb, const Lane& L, float inv, uint32_t (&qsw)[2][4], uint32_t (&QH)[2][2],
                              uint32_t (&sgw)[2][4], float (&db)[2]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t r8 = sb + L.row8c + h * L.rb8, r4 = sb + L.row4c + h * L.rb8;
        const uint32_t r1 = sb + L.row1c + h * L.rb8, rh = sb + L.rowhc + h * L.rb8;
        const float d = __half2float(__ushort_as_half((unsigned short)ld_u16<0>(sb + L.row0 + h * L.rb8)));
        qsw[h][0] = ld_u16<2 + 32 * N>(r8);
        qsw[h][1] = ld_u16<4 + 32 * N>(r8);
        qsw[h][2] = ld_u16<6 + 32 * N>(r8);
        qsw[h][3] = ld_u16<8 + 32 * N>(r8);
        sgw[h][0] = ld_u8<74 + 16 * N>(r4);
        sgw[h][1] = ld_u8<75 + 16 * N>(r4);
        sgw[h][2] = ld_u8<76 + 16 * N>(r4);
        sgw[h][3] = ld_u8<77 + 16 * N>(r4);
        const uint32_t qh = ld_u8<66 + 4 * N>(r1);
        QH[h][0] = ((qh & 15u) * 0x00204081u) & 0x01010101u;   // qh bits 0..3 -> bytes 0..3
        QH[h][1] = ((qh >> 4) * 0x00204081u) & 0x01010101u;    // qh bits 4..7 -> bytes 0..3
        const uint32_t nib = (ld_u8<106 + 2 * N>(rh) >> L.nib_shift) & 15u;
        db[h] = d * (float)(1 + 2 * (int)nib) * inv;
    }
}

// Step S (grid entry S of the lane's sub-block) for rows g and g + 8: decode
// into A fragments and issue the MMA into accumulator S & 1.
template <int S>
__device__ inline void step1(uint32_t table, const uint32_t (&qsw)[2][4], const uint32_t (&QH)[2][2],
                             const uint32_t (&sgw)[2][4], const uint32_t (&bf)[8][2], float (&dd)[2][4]) {
    uint32_t a[2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) decode_entry<S>(qsw[h][S >> 1], QH[h][S >> 2], sgw[h][S >> 1], table, a[h][0], a[h][1]);
    mma16816(dd[S & 1], a[0][0], a[1][0], a[0][1], a[1][1], bf[S][0], bf[S][1]);
}

// One 128-weight group (sub-blocks 4N .. 4N + 3 of the super-block at sb) of a
// 16-row tile: adds the dots of rows g and g + 8 (this lane's sub-block) to acc.
template <int N>
__device__ inline void do_group(uint32_t sb, const Lane& L, uint32_t tab, const uint32_t (&bf)[8][2], float inv,
                                float (&acc)[2]) {
    uint32_t qsw[2][4], QH[2][2], sgw[2][4];
    float db[2];
    fields<N>(sb, L, inv, qsw, QH, sgw, db);
    float dd[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    step1<0>(tab, qsw, QH, sgw, bf, dd);
    step1<1>(tab, qsw, QH, sgw, bf, dd);
    step1<2>(tab, qsw, QH, sgw, bf, dd);
    step1<3>(tab, qsw, QH, sgw, bf, dd);
    step1<4>(tab, qsw, QH, sgw, bf, dd);
    step1<5>(tab, qsw, QH, sgw, bf, dd);
    step1<6>(tab, qsw, QH, sgw, bf, dd);
    step1<7>(tab, qsw, QH, sgw, bf, dd);
    acc[0] = fmaf(db[0], (dd[0][0] + dd[0][1]) + (dd[1][0] + dd[1][1]), acc[0]);
    acc[1] = fmaf(db[1], (dd[0][2] + dd[0][3]) + (dd[1][2] + dd[1][3]), acc[1]);
}

// group q of a row: super-block q / 2, half q % 2
__device__ inline void do_group_q(uint32_t tile, int q, const Lane& L, uint32_t tab, const uint32_t (&bf)[8][2], float inv,
                                  float (&acc)[2]) {
    const uint32_t sb = tile + (uint32_t)(q >> 1) * 110u;
    if (q & 1)
        do_group<1>(sb, L, tab, bf, inv, acc);
    else
        do_group<0>(sb, L, tab, bf, inv, acc);
}

// Step S for the same group of two tiles: four independent entry chains and
// two MMA chains, sharing the B fragments.
template <int S>
__device__ inline void step2(uint32_t table, const uint32_t (&qsw)[2][2][4], const uint32_t (&QH)[2][2][2],
                             const uint32_t (&sgw)[2][2][4], const uint32_t (&bf)[8][2], float (&dd)[2][4]) {
    uint32_t a[2][2][2];
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h)
            decode_entry<S>(qsw[t][h][S >> 1], QH[t][h][S >> 2], sgw[t][h][S >> 1], table, a[t][h][0], a[t][h][1]);
#pragma unroll
    for (int t = 0; t < 2; ++t)
        mma16816(dd[t], a[t][0][0], a[t][1][0], a[t][0][1], a[t][1][1], bf[S][0], bf[S][1]);
}

// Group 4N .. 4N + 3 of the super-blocks at sb0 and sb1 (two tiles, same
// offsets): acc0 / acc1 get rows g and g + 8 of each.
template <int N>
__device__ inline void do_group2(uint32_t sb0, uint32_t sb1, const Lane& L, uint32_t tab, const uint32_t (&bf)[8][2],
                                 float inv, float (&acc0)[2], float (&acc1)[2]) {
    uint32_t qsw[2][2][4], QH[2][2][2], sgw[2][2][4];
    float db[2][2];
    fields<N>(sb0, L, inv, qsw[0], QH[0], sgw[0], db[0]);
    fields<N>(sb1, L, inv, qsw[1], QH[1], sgw[1], db[1]);
    float dd[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    step2<0>(tab, qsw, QH, sgw, bf, dd);
    step2<1>(tab, qsw, QH, sgw, bf, dd);
    step2<2>(tab, qsw, QH, sgw, bf, dd);
    step2<3>(tab, qsw, QH, sgw, bf, dd);
    step2<4>(tab, qsw, QH, sgw, bf, dd);
    step2<5>(tab, qsw, QH, sgw, bf, dd);
    step2<6>(tab, qsw, QH, sgw, bf, dd);
    step2<7>(tab, qsw, QH, sgw, bf, dd);
    acc0[0] = db[0][0] * (dd[0][0] + dd[0][1]);
    acc0[1] = db[0][1] * (dd[0][2] + dd[0][3]);
    acc1[0] = db[1][0] * (dd[1][0] + dd[1][1]);
    acc1[1] = db[1][1] * (dd[1][2] + dd[1][3]);
}

__device__ inline void do_group2_q(uint32_t tile0, uint32_t tile1, int q, const Lane& L, uint32_t tab,
                                   const uint32_t (&bf)[8][2],
                                   float inv, float (&acc0)[2], float (&acc1)[2]) {
    const uint32_t o = (uint32_t)(q >> 1) * 110u;
    if (q & 1)
        do_group2<1>(tile0 + o, tile1 + o, L, tab, bf, inv, acc0, acc1);
    else
        do_group2<0>(tile0 + o, tile1 + o, L, tab, bf, inv, acc0, acc1);
}

// Both groups (sub-blocks 0-3 and 4-7) of the super-block at sb of one
// 16-row tile, with each group's B staged in shared memory (bst0, bst1) and
// its own scale: two independent MMA chains; acc gets rows g and g + 8.
template <int S>
__device__ inline void step_sb(uint32_t table, const uint32_t (&qsw)[2][2][4], const uint32_t (&QH)[2][2][2],
                               const uint32_t (&sgw)[2][2][4], uint32_t bst0, uint32_t bst1, float (&dd)[2][4]) {
    uint32_t a[2][2][2];
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
        for (int h = 0; h < 2; ++h)
            decode_entry<S>(qsw[n][h][S >> 1], QH[n][h][S >> 2], sgw[n][h][S >> 1], table, a[n][h][0], a[n][h][1]);
    uint32_t b[2][2];
    load_b(bst0, S, b[0][0], b[0][1]);
    load_b(bst1, S, b[1][0], b[1][1]);
#pragma unroll
    for (int n = 0; n < 2; ++n) mma16816(dd[n], a[n][0][0], a[n][1][0], a[n][0][1], a[n][1][1], b[n][0], b[n][1]);
}

__device__ inline void do_superblock(uint32_t sb, const Lane& L, uint32_t tab, uint32_t bst0, float inv0, uint32_t bst1,
                                     float inv1, float (&acc)[2]) {
    uint32_t qsw[2][2][4], QH[2][2][2], sgw[2][2][4];
    float db[2][2];
    fields<0>(sb, L, inv0, qsw[0], QH[0], sgw[0], db[0]);
    fields<1>(sb, L, inv1, qsw[1], QH[1], sgw[1], db[1]);
    float dd[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    step_sb<0>(tab, qsw, QH, sgw, bst0, bst1, dd);
    step_sb<1>(tab, qsw, QH, sgw, bst0, bst1, dd);
    step_sb<2>(tab, qsw, QH, sgw, bst0, bst1, dd);
    step_sb<3>(tab, qsw, QH, sgw, bst0, bst1, dd);
    step_sb<4>(tab, qsw, QH, sgw, bst0, bst1, dd);
    step_sb<5>(tab, qsw, QH, sgw, bst0, bst1, dd);
    step_sb<6>(tab, qsw, QH, sgw, bst0, bst1, dd);
    step_sb<7>(tab, qsw, QH, sgw, bst0, bst1, dd);
    acc[0] = fmaf(db[0][0], dd[0][0] + dd[0][1], db[1][0] * (dd[1][0] + dd[1][1]));
    acc[1] = fmaf(db[0][1], dd[0][2] + dd[0][3], db[1][1] * (dd[1][2] + dd[1][3]));
}

// rows g, g + 8 of the quad's partial sums, summed over the quad (c = 0..3)
__device__ inline void quad_sum(float (&acc)[2]) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 1);
        acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 2);
    }
}

}  // namespace sb_flow
