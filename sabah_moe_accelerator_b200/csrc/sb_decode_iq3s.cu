// Persistent IQ3_S decode: every layer of a decode step in ONE cooperative
// launch, one CTA per SM (sabah_moe_decode's fast path).
//
// A step is 2 * n_layers phases: gate/up of layer L, then down + top-k combine
// + residual of layer L. The per-launch kernels of sb_mmid_iq3s.cu pay, per
// phase, a launch, a CTA ramp-up, a grid-table fill, a cold weight pipeline and
// a tail; here all of that is paid once per step:
//
// * The producer warp walks this CTA's items of ALL phases in order and never
//   waits for a phase boundary: weights and router ids are inputs, so it streams
//   the next phase's tiles into the stage ring while the consumers finish the
//   current phase and wait at the grid barrier.
// * Consumers wait at a grid barrier before each phase, then build the
//   x-fragment sets of the phase's input vectors: x (gate/up) or h (down).
// * Work is cut into units that a CTA owns whole, so every combine is local:
//   a gate/up unit is 32 rows (one IQ3_S sub-block of h) of one (token, slot):
//   its two gate and two up 16-row tiles - four items - whose last item writes
//   h = silu(g) * u and, since it holds a whole sub-block, the sub-block's
//   x-fragment record of the down phase's set straight to global memory; the
//   down phase then fetches a token's sets with one bulk copy. A down unit is
//   16 rows of one token over all n_used slots, two slots per item (two bulk
//   copies into one stage), whose last item sums the slots in slot order from
//   shared memory and updates x in place (x += sum_e w_e v_e).
// * The decode core (grid lookup + PRMT into fp16 subnormals + mma.sync) is
//   the one of sb_mmid_iq3s.cu.
//
// Every wait is bounded (stage barriers, sequence stamps, the grid barrier); a
// CTA that gives up records SB_DERR_TIMEOUT, skips its remaining work, still
// arrives at every grid barrier and drains its copies before it exits.
#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "sb_iq3s_core.cuh"

namespace {

using namespace sb_iq3s;

constexpr int kNC = 16;                      // consumer warps
#ifndef SB_DECODE_LOG_R
#define SB_DECODE_LOG_R 5
#endif
constexpr int kLogR = SB_DECODE_LOG_R;       // grid-table replicas: 32, conflict-free lookups
constexpr int kR = 1 << kLogR;
constexpr int kThreads = (kNC + 1) * 32;     // + one producer warp
constexpr int kStageBytes = 16 * 880;        // a 16-row tile at k <= 2048, or two at k <= 1024
constexpr int kStages = 8;                   // = kIssuers: producer lane l owns stage l
constexpr int kSetArea = 4 * kSetBytes;      // x-fragment sets of one chunk
constexpr int kGuSets = 4;                   // gate/up: token vectors per chunk
constexpr int kMaxWpt = 4;
constexpr int kMaxLayers = 64;
constexpr int kMaxUsed = 16;
constexpr int kUnits = 4;                    // down units with a combine buffer
constexpr long long kBarPolls = 1ll << 22;   // grid-barrier polls
static_assert(kStages % kIssuers == 0, "a stage must always belong to the same producer lane");

struct Desc {
    int seq;       // sequence number of the tile(s) in the stage
    int bad;       // 0 valid, else the device error code
    int slot;      // x-fragment set of tile 0 (tile 1 uses slot + 1)
    int t, e, rt;  // token, slot (gate/up) or first slot (down), 16-row tile
    int which;     // gate/up: 0 gate, 1 up
    int n;         // down: tiles present (1 when n_used is odd and this is the last pair)
};

struct Smem {
    static constexpr int table = 0;
    static constexpr int stages = table + table_bytes<kR>();
    static constexpr int sets = stages + kStages * kStageBytes;
    static constexpr int red = sets + kSetArea;                        // [kStages][kMaxWpt][32] floats
    static constexpr int ubuf = red + kStages * kMaxWpt * 32 * 4;      // [kUnits][kMaxUsed][16] floats
    static constexpr int desc = ubuf + kUnits * kMaxUsed * 16 * 4;     // [kStages] Desc
    static constexpr int cnt = desc + kStages * (int)sizeof(Desc);     // [kStages] ints
    static constexpr int ucnt = cnt + kStages * 4;                     // [kUnits] ints
    static constexpr int ugen = ucnt + kUnits * 4;                     // [kUnits] ints
    static constexpr int abort_flag = ugen + kUnits * 4;
    static constexpr int bars = (abort_flag + 4 + 7) & ~7;             // full[kStages], empty[kStages], set
    static constexpr int total = bars + (2 * kStages + 1) * 8;
};
static_assert(Smem::total <= 227 * 1024, "shared memory budget");
static_assert(Smem::stages % 128 == 0 && kStageBytes % 128 == 0, "stage alignment");

// One phase kind's geometry. A task is one super-block pair (256 weights) of
// one 16-row tile; an item has n_tiles * ppr tasks, split over wpt warps.
struct Geo {
    int n_items;     // items per phase
    int per_key;     // items per token
    int per_unit;    // items per unit
    int rtiles;      // 16-row tiles per matrix
    int n_tiles;     // 16-row tiles per item (1 gate/up, 2 down)
    int ppr;         // super-block pairs per row (k / 256)
    int wpt, tpw;    // warps per item, tasks per warp
    int k, rb;       // row length, row bytes
    int set_stride;  // bytes of one x-fragment set (k / 128 groups)
    int rowpair;     // down with one slot: an item is 32 rows (two row tiles) of that slot
};

struct LayerBanks {
    const uint8_t* gate;
    const uint8_t* up;
    const uint8_t* down;
    const int32_t* ids;   // [T][n_used]
    const float* w;       // [T][n_used]
};

struct DecodeParams {
    Geo gu, dn;
    int n_layers, n_tokens, n_used, n_experts, d_model, ff;
    size_t gu_stride, dn_stride;   // bytes between experts
    float* x;                      // [T][d_model]: the blocks' input (x += block(x) per layer when out == x)
    float* out;                    // the combine's destination: out = (accumulate ? out : 0) + y
    int accumulate;
    const int32_t* xrows;          // one block: token t's input is row xrows[t] of x (nullptr: row t)
    int n_xrows;
    float* h;                      // [T][n_used][ff]
    uint8_t* hsets;                // [T][n_used] down-phase x-fragment sets of h (dn.set_stride bytes each)
    unsigned* sync;                // [0] grid-barrier arrivals, [1] exits; reset by the last CTA to exit
    int* err;
    LayerBanks layer[kMaxLayers];
};

__device__ inline void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kNC * 32) : "memory"); }

__device__ inline unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// The 16-row tile rt of the expert routed at (token, slot) si; kind 0 gate,
// 1 up, 2 down; nullptr for an id outside [0, n_experts).
__device__ inline const uint8_t* expert_row_tile(const DecodeParams& p, const LayerBanks& lb, int kind, int si, int rt,
                                                 int e) {
    int id = lb.ids[si];
#if SABAH_SENTINEL == 1
    if (e == 0 && id >= 0 && id < p.n_experts) id = (id + 1) % p.n_experts;   // test-only build
#endif
    if (id < 0 || id >= p.n_experts) return nullptr;
    const uint8_t* base = kind == 2 ? lb.down : kind == 1 ? lb.up : lb.gate;
    const size_t stride = kind == 2 ? p.dn_stride : p.gu_stride;
    const int rb = kind == 2 ? p.dn.rb : p.gu.rb;
    return base + (size_t)id * stride + (size_t)rt * 16 * rb;
}

// this CTA's items of a phase: whole units, split evenly
__device__ inline void phase_range(const DecodeParams& p, bool down, int& i0, int& i1) {
    const Geo& G = down ? p.dn : p.gu;
    const int n = G.n_items / G.per_unit;
    i0 = (int)((long long)blockIdx.x * n / gridDim.x) * G.per_unit;
    i1 = (int)((long long)(blockIdx.x + 1) * n / gridDim.x) * G.per_unit;
}

// Lane l of a warp holds element l of sub-block j of a vector; the warp writes
// the sub-block's x-fragment record into the vector's set at `set` (global),
// exactly as set_put builds it in shared memory: per-sub-block power-of-two
// scale, fp16 hi and lo parts, records (j / 4, step s) at quad j % 4, the zero
// pairs (by quad 0) and the inverse scale.
__device__ inline void put_record(float v, int lane, int j, uint8_t* set) {
    float m = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int ex = 0;
    if (m > 0.f && isfinite(m)) {
        frexpf(m, &ex);   // m = f * 2^ex, f in [0.5, 1)
        ex = max(-100, min(100, 14 - ex));
    }
    const float s = ldexpf(1.f, ex);
    const float vs = v * s;
    const __half hi = __float2half_rn(vs), lo = __float2half_rn(vs - __half2float(hi));
    // pairs (2i, 2i + 1) into even lanes, then elements 4s+2, 4s+3 into lane 4s
    const uint32_t hb = __half_as_ushort(hi), lb = __half_as_ushort(lo);
    const uint32_t hp = hb | (__shfl_xor_sync(0xffffffffu, hb, 1) << 16);
    const uint32_t lp = lb | (__shfl_xor_sync(0xffffffffu, lb, 1) << 16);
    const uint32_t hp23 = __shfl_down_sync(0xffffffffu, hp, 2), lp23 = __shfl_down_sync(0xffffffffu, lp, 2);
    const int q = j >> 2, c = j & 3, st = lane >> 2;
    uint8_t* grp = set + q * kGroupBytes;
    if ((lane & 3) == 0) {
        uint2* rec = (uint2*)(grp + st * kRecBytes);
        rec[2 * c] = make_uint2(hp, hp23);
        rec[2 * c + 1] = make_uint2(lp, lp23);
        if (c == 0) rec[8] = make_uint2(0, 0);
    }
    // 2^24 undoes the subnormal encoding of the weights, 1/s the x scale
    if (lane == 0) ((float*)(grp + 8 * kRecBytes))[c] = 16777216.0f / s;
}

__global__ void __launch_bounds__(kThreads, 1) k_decode_iq3s(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bars = (uint64_t*)(smem + Smem::bars);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStages), setbar = smem_u32(bars + 2 * kStages);
    volatile int* abort_flag = (volatile int*)(smem + Smem::abort_flag);
    Desc* descs = (Desc*)(smem + Smem::desc);
    const int n_phases = 2 * p.n_layers;

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);   // one release per item, by its last warp
        }
        mbar_init(setbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (threadIdx.x < kStages) {
        ((int*)(smem + Smem::cnt))[threadIdx.x] = 0;
        descs[threadIdx.x].seq = -1;
    }
    __syncthreads();

    if (warp == kNC) {
        // ------------------------------------------------------ producer
        // lane l issues the sequence numbers n = l, l + 8, ... of this CTA's
        // items over all phases, always into stage n % 8 = l
        if (lane < kIssuers) {
            const uint32_t st0 = smem_u32(smem + Smem::stages);
            int n = 0, last = -1;
            bool stop = false;
            for (int ph = 0; ph < n_phases && !stop; ++ph) {
                const bool down = ph & 1;
                const Geo& G = down ? p.dn : p.gu;
                const LayerBanks& lb = p.layer[ph >> 1];
                int i0, i1;
                phase_range(p, down, i0, i1);
                for (int item = i0; item < i1; ++item, ++n) {
                    if (n % kIssuers != lane) continue;
                    if (*abort_flag) {
                        stop = true;
                        break;
                    }
                    const int s = n % kStages;
                    if (n >= kStages && !mbar_wait(empty0 + 8 * s, ((n / kStages) - 1) & 1, p.err, abort_flag)) {
                        stop = true;
                        break;
                    }
                    Desc d;
                    const uint8_t* src[2] = {nullptr, nullptr};
                    d.bad = 0;
                    if (!down) {
                        // unit (token, slot, 32-row block): gate 0-15, up 0-15, gate 16-31, up 16-31
                        const int unit = item >> 2, part = item & 3;
                        d.which = part & 1;
                        const int si = unit / (G.rtiles / 2);
                        d.rt = 2 * (unit % (G.rtiles / 2)) + (part >> 1);
                        d.t = si / p.n_used;
                        d.e = si % p.n_used;
                        d.n = 1;
                        d.slot = d.t % kGuSets;
                        src[0] = expert_row_tile(p, lb, d.which, si, d.rt, d.e);
                    } else {
                        d.which = 0;
                        if (G.rowpair) {
                            // one slot: the unit (and item) is 32 rows, row tiles 2rb and 2rb + 1
                            d.t = item / (G.rtiles / 2);
                            d.rt = 2 * (item % (G.rtiles / 2));
                            d.e = 0;
                            d.n = 2;
                            d.slot = 0;
                            for (int tl = 0; tl < 2; ++tl)
                                src[tl] = expert_row_tile(p, lb, 2, d.t * p.n_used, d.rt + tl, 0);
                        } else {
                            const int unit = item / G.per_unit, pair = item % G.per_unit;
                            d.t = unit / G.rtiles;
                            d.rt = unit % G.rtiles;
                            d.e = 2 * pair;
                            d.n = min(2, p.n_used - d.e);
                            d.slot = d.e;
                            for (int tl = 0; tl < d.n; ++tl)
                                src[tl] = expert_row_tile(p, lb, 2, d.t * p.n_used + d.e + tl, d.rt, d.e + tl);
                        }
                    }
                    for (int tl = 0; tl < d.n; ++tl)
                        if (!d.bad) d.bad = !src[tl] ? SB_DERR_BAD_ID : ((uintptr_t)src[tl] & 15) ? SB_DERR_MISALIGNED : 0;
                    d.seq = -1;
                    descs[s] = d;
                    __threadfence_block();
                    *(volatile int*)&descs[s].seq = n;   // the stage's previous tile is released
                    if (!d.bad) {
                        const uint32_t tb = 16u * G.rb;
                        mbar_expect_tx(full0 + 8 * s, tb * d.n);
                        for (int tl = 0; tl < d.n; ++tl)
                            bulk_g2s(st0 + s * kStageBytes + tl * tb, src[tl], tb, full0 + 8 * s);
                    } else {
                        mbar_arrive(full0 + 8 * s);
                    }
                    last = n;
                }
            }
            // never leave with a copy in flight: the last use of this lane's stage must have landed
            if (last >= 0)
                for (long long i = 0; i < kSpinLimit && !mbar_try_wait(full0 + 8 * (last % kStages),
                                                                       (last / kStages) & 1); ++i) {
                }
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    uint32_t* table = (uint32_t*)(smem + Smem::table);
    fill_table<kNC * 32, kR>(table);
    const int g = lane >> 2, c = lane & 3;
    const uint32_t boff = lane_boff(lane);
    const uint32_t stages32 = smem_u32(smem + Smem::stages), sets32 = smem_u32(smem + Smem::sets);
    float* red = (float*)(smem + Smem::red);
    float* ubuf = (float*)(smem + Smem::ubuf);
    int* cnt = (int*)(smem + Smem::cnt);
    int* ucnt = (int*)(smem + Smem::ucnt);
    volatile int* ugen = (volatile int*)(smem + Smem::ugen);
    uint8_t* sets = smem + Smem::sets;
    const DecodeParams* pp = &p;
    int seq_base = 0;
    int set_copies = 0;   // bulk copies of down-phase sets issued (thread 0) and waited for

    for (int ph = 0; ph < n_phases; ++ph) {
        // grid barrier: the previous phase's rows (or x) are all written
        consumers_sync();
        if (ph > 0 && threadIdx.x == 0) {
            // release: the CTA's writes (ordered before by the bar.sync) become
            // visible with the arrival; acquire: other CTAs' writes are visible
            // to this CTA after the wait (and to its other threads after the bar.sync)
            asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.sync) : "memory");
            const unsigned target = (unsigned)ph * gridDim.x;
            bool ok = *abort_flag != 0;   // an aborting CTA still arrives, but does not wait
            for (long long i = 0; i < kBarPolls && !ok; ++i) ok = ld_acquire(p.sync) >= target;
            if (!ok) {
                *abort_flag = 1;
                if (p.err) atomicExch(p.err, SB_DERR_TIMEOUT);
            }
        }
        if (threadIdx.x < kUnits) {   // every unit of the previous down phase is complete
            ucnt[threadIdx.x] = 0;
            ugen[threadIdx.x] = 0;
        }
        consumers_sync();
        const int layer = ph >> 1;
        const bool down = ph & 1;
        const Geo& G = down ? p.dn : p.gu;
        int i0, i1;
        phase_range(p, down, i0, i1);
        const Lane L = lane_init<kR>(table, G.rb, lane);
        const int P = kNC / G.wpt;
        const int pos = warp / G.wpt, wsub = warp % G.wpt;

        int item = i0;
        while (item < i1) {
            // chunk: gate/up up to kGuSets tokens; down one token (its n_used slots)
            int chunk_end, key0, n_keys;
            if (!down) {
                key0 = item / G.per_key;
                chunk_end = min(i1, (key0 + kGuSets) * G.per_key);
                n_keys = (chunk_end - 1) / G.per_key - key0 + 1;
            } else {
                const int t = item / G.per_key;
                chunk_end = min(i1, (t + 1) * G.per_key);
                key0 = t * p.n_used;
                n_keys = p.n_used;
            }
            if (item > i0) consumers_sync();   // every warp is done with the previous chunk's sets
            const int sst = G.set_stride;
            if (down) {
                // the token's n_used sets, written by the gate/up units, in one bulk copy.
                // The generic-proxy writes of other CTAs (released at the grid barrier,
                // acquired by thread 0) are ordered before this async-proxy read, and the
                // set area's earlier generic reads before its overwrite, by the proxy fence.
                if (threadIdx.x == 0) {
                    asm volatile("fence.proxy.async;" ::: "memory");
                    const uint32_t bytes = (uint32_t)(n_keys * sst);
                    mbar_expect_tx(setbar, bytes);
                    bulk_g2s(sets32, p.hsets + (size_t)key0 * sst, bytes, setbar);
                }
                mbar_wait(setbar, set_copies & 1, p.err, abort_flag);   // on timeout the items see the abort
                ++set_copies;
            } else {
                build_sets_from<kNC * 32>(
                    n_keys,
                    [pp, key0](int i, int f) {
                        int r = key0 + i;
                        if (pp->xrows) {
                            r = __ldg(pp->xrows + r);
                            if (r < 0 || r >= pp->n_xrows) {   // no such row: NaN outputs, error recorded
                                if (f == 0 && pp->err) atomicExch(pp->err, SB_DERR_BAD_ID);
                                const float nan = __int_as_float(0x7fc00000);
                                return make_float4(nan, nan, nan, nan);
                            }
                        }
                        return __ldcg((const float4*)(pp->x + (size_t)r * pp->d_model) + f);
                    },
                    [sets, sst, key0](int i) { return sets + ((key0 + i) % kGuSets) * sst; }, G.k);
            }
            consumers_sync();
            for (int it = item + pos; it < chunk_end; it += P) {
                const int seq = seq_base + (it - i0);
                const int s = seq % kStages;
                const bool stamped = wait_seq(&descs[s].seq, seq, p.err, abort_flag);
                const bool landed = stamped && mbar_wait(full0 + 8 * s, (seq / kStages) & 1, p.err, abort_flag);
                const Desc d = descs[s];
                const int bad = !stamped ? -1 : !landed ? SB_DERR_TIMEOUT : d.bad;
                float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
                if (!bad) {
                    const uint32_t tile0 = stages32 + s * kStageBytes;
                    for (int j = wsub * G.tpw; j < (wsub + 1) * G.tpw; ++j) {
                        const int tl = j / G.ppr, q = 2 * (j - tl * G.ppr);
                        if (tl >= d.n) break;
                        float r[2] = {0.f, 0.f};
                        const int set = d.slot + (G.rowpair ? 0 : tl);
                        do_pair<kLogR>(tile0 + (uint32_t)(tl * 16 * G.rb), q, sets32 + set * sst + boff, L, r);
                        acc[0][0] += tl ? 0.f : r[0];
                        acc[0][1] += tl ? 0.f : r[1];
                        acc[1][0] += tl ? r[0] : 0.f;
                        acc[1][1] += tl ? r[1] : 0.f;
                    }
                }
#pragma unroll
                for (int tl = 0; tl < 2; ++tl)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        acc[tl][h] += __shfl_xor_sync(0xffffffffu, acc[tl][h], 1);
                        acc[tl][h] += __shfl_xor_sync(0xffffffffu, acc[tl][h], 2);
                    }
                float* rr = red + (s * kMaxWpt + wsub) * 32;
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
                    last = atomicAdd(cnt + s, 1) == G.wpt - 1;
                    if (last) cnt[s] = 0;
                }
                last = __shfl_sync(0xffffffffu, last, 0);
                if (!last) continue;
                // ---- epilogue (the last warp of the item): sum the warps' rows in fixed order
                __threadfence_block();
                float v = 0.f;
                for (int w = 0; w < G.wpt; ++w) v += red[(s * kMaxWpt + w) * 32 + lane];
                __syncwarp();
                // the partial rows are read: the stage (and its red slot) may be reused
                if (lane == 0) mbar_arrive(empty0 + 8 * s);
                if (bad < 0) continue;   // no descriptor (the CTA is aborting; the error is recorded)
                if (bad > 0) {
                    v = __int_as_float(0x7fc00000);
                    if (lane == 0 && p.err) atomicExch(p.err, bad);
                }
                // The item's rows go to its unit's buffer; the unit's last item
                // combines them. Buffer ub serves this CTA's units ub, ub + kUnits,
                // ...: an item first waits until the buffer's previous unit is done
                // (its generation). The earliest unfinished unit never waits, and a
                // waiting warp holds no stage, so the wait always ends.
                const int lu = (it - i0) / G.per_unit;
                const int ub = lu % kUnits, gen = lu / kUnits;
                if (lane == 0) {
                    bool ok = ugen[ub] == gen;
                    for (long long i = 0; i < kSpinLimit * 64 && !ok && !*abort_flag; ++i) {
                        __nanosleep(64);
                        ok = ugen[ub] == gen;
                    }
                    if (!ok && !*abort_flag) {
                        *abort_flag = 1;
                        if (p.err) atomicExch(p.err, SB_DERR_TIMEOUT);
                    }
                }
                __syncwarp();
                __threadfence_block();
                float* ubase = ubuf + ub * kMaxUsed * 16;
                if (!down) {
                    if (lane < 16) ubase[(d.which * 2 + (d.rt & 1)) * 16 + lane] = v;   // gate rows, up rows
                } else {
                    // row pair: buffer rows 0..31 of the single slot; else 16 rows per slot
                    const int tl = lane >> 4, e = G.rowpair ? d.e : d.e + tl;
                    if (tl < d.n)
                        ubase[(G.rowpair ? tl : e) * 16 + (lane & 15)] = __ldg(p.layer[layer].w + d.t * p.n_used + e) * v;
                }
                __threadfence_block();
                __syncwarp();
                int ulast = 0;
                if (lane == 0) {
                    ulast = atomicAdd(ucnt + ub, 1) == G.per_unit - 1;
                    if (ulast) ucnt[ub] = 0;
                }
                ulast = __shfl_sync(0xffffffffu, ulast, 0);
                if (!ulast) continue;
                __threadfence_block();
                if (!down) {
                    // h of the unit's 32 rows (one sub-block), then its set record
                    const size_t si = (size_t)d.t * p.n_used + d.e;
                    const int half = lane >> 4, r16 = lane & 15, j = d.rt >> 1;
                    const float gv = ubase[half * 16 + r16], uv = ubase[(2 + half) * 16 + r16];
                    const float hv = gv / (1.f + expf(-gv)) * uv;
                    p.h[si * p.ff + 32 * j + lane] = hv;
                    put_record(hv, lane, j, p.hsets + si * p.dn.set_stride);
                } else if (G.rowpair) {
                    // one slot, 32 rows
                    const float tot = ubase[lane];
                    float* o = p.out + (size_t)d.t * p.d_model + d.rt * 16 + lane;
                    *o = p.accumulate ? __ldcg(o) + tot : tot;
                } else if (lane < 16) {
                    // the top-k weighted sum in slot order, then the residual
                    float tot = 0.f;
                    for (int e2 = 0; e2 < p.n_used; ++e2) tot += ubase[e2 * 16 + lane];
                    float* o = p.out + (size_t)d.t * p.d_model + d.rt * 16 + lane;
                    *o = p.accumulate ? __ldcg(o) + tot : tot;
                }
                __syncwarp();
                __threadfence_block();
                if (lane == 0) ugen[ub] = gen + 1;   // the buffer is free for the next unit
            }
            item = chunk_end;
        }
        seq_base += i1 - i0;
    }
    // never leave with a set copy in flight (its wait may have given up)
    if (threadIdx.x == 0 && set_copies > 0)
        for (long long i = 0; i < kSpinLimit && !mbar_try_wait(setbar, (set_copies - 1) & 1); ++i) {
        }
    // the last CTA out resets the barrier words for the next launch
    consumers_sync();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(p.sync + 1, 1u) == gridDim.x - 1) {
            p.sync[0] = 0;
            p.sync[1] = 0;
            __threadfence();
        }
    }
}

// ------------------------------------------------------------------ host side
// Geometry of a phase kind with n_tiles 16-row tiles per item.
bool plan(int k, int rows, int n_tiles, Geo& G) {
    if (k % 256 || k > 2048 || rows % 16) return false;
    G.k = k;
    G.rb = (int)sb_row_bytes_of(SB_IQ3_S, k);
    if (n_tiles * 16 * G.rb > kStageBytes || (16 * G.rb) % 16) return false;
    G.n_tiles = n_tiles;
    G.ppr = k / 256;
    G.rtiles = rows / 16;
    G.set_stride = (k / 128) * kGroupBytes;
    const int tasks = G.n_tiles * G.ppr;
    G.wpt = 1;
    for (int w : {4, 2})
        if (tasks % w == 0) {
            G.wpt = w;
            break;
        }
    G.tpw = tasks / G.wpt;
    return true;
}

struct DecodeScratch {
    void* mem = nullptr;
    size_t counter_cap = 0, partial_cap = 0;
    bool stale = false;
};
DecodeScratch g_ds;
// launch attribute and grid, per device (the smem opt-in is a per-device setting)
constexpr int kMaxDev = 64;
bool g_attr_set[kMaxDev] = {};
int g_grid[kMaxDev] = {};

bool fast_path_enabled() {
    static int on = -1;
    if (on < 0) {
        const char* v = std::getenv("SABAH_IQ3S_PERSISTENT");
        const char* m = std::getenv("SABAH_IQ3S_MMA");
        on = !(v && *v == '0') && !(m && *m == '0');
    }
    return on != 0;
}

}  // namespace

void sb_decode_scratch_invalidate() {
    g_ds.stale = g_ds.mem != nullptr;
    sb_flow_scratch_invalidate();
}

int sb_try_decode_iq3s(const sb_decode_args& a, cudaStream_t st) {
    if (a.qt_gate != SB_IQ3_S || a.qt_up != SB_IQ3_S || a.qt_down != SB_IQ3_S || !fast_path_enabled()) return 0;
    // one token: the barrier-free kernel (sb_flow_iq3s.cu); more tokens, gathered
    // rows or shapes it does not cover: the phase-barrier kernel below
    const int flow = sb_try_flow_iq3s(a, st);
    if (flow != 0) return flow;
    if (a.n_layers < 1 || a.n_layers > kMaxLayers || a.n_tokens < 1 || a.n_used < 1 || a.n_used > kMaxUsed) return 0;
    DecodeParams p{};
    if (!plan(a.d_model, a.ff, 1, p.gu) || !plan(a.ff, a.d_model, 2, p.dn)) return 0;
    if (kGuSets * p.gu.set_stride > kSetArea || a.n_used * p.dn.set_stride > kSetArea) return 0;
    if (a.gu_expert_stride % 16 || a.down_expert_stride % 16 || ((uintptr_t)a.x & 15) || !a.out) return 0;
    if (a.n_layers > 1 && (a.out != a.x || !a.accumulate || a.xrows)) return 0;   // the residual chain
    if ((long long)a.n_tokens * a.n_used > 16384) return 0;
    for (int L = 0; L < a.n_layers; ++L)
        for (const void* b : {a.gate_banks[L], a.up_banks[L], a.down_banks[L]})
            if (!b || ((uintptr_t)b & 15)) return 0;
    const long long gu_items = (long long)a.n_tokens * a.n_used * p.gu.rtiles * 2;
    const int pairs = (a.n_used + 1) / 2;
    p.dn.rowpair = a.n_used == 1 && p.dn.rtiles % 2 == 0;
    const long long dn_items = p.dn.rowpair ? (long long)a.n_tokens * (p.dn.rtiles / 2)
                                            : (long long)a.n_tokens * p.dn.rtiles * pairs;
    if (gu_items > (1 << 28) || dn_items > (1 << 28)) return 0;
    if (((uintptr_t)a.h & 15)) return 0;
    p.gu.n_items = (int)gu_items;
    p.gu.per_key = a.n_used * p.gu.rtiles * 2;   // items of one token
    p.gu.per_unit = 4;                           // gate and up tiles of 32 rows (one sub-block of h)
    p.dn.n_items = (int)dn_items;
    p.dn.per_key = p.dn.rowpair ? p.dn.rtiles / 2 : p.dn.rtiles * pairs;   // items of one token
    p.dn.per_unit = p.dn.rowpair ? 1 : pairs;    // 32 rows of one slot, or 16 rows over all slots

    int dev = 0;
    if (!sb_cuda_ok(cudaGetDevice(&dev), "decode device")) return -1;
    if (dev < 0 || dev >= kMaxDev) return 0;
    if (!g_attr_set[dev]) {
        if (!sb_cuda_ok(cudaFuncSetAttribute(k_decode_iq3s, cudaFuncAttributeMaxDynamicSharedMemorySize, Smem::total),
                        "decode smem attribute"))
            return -1;
        int sms = 0, per_sm = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (!sb_cuda_ok(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode_iq3s, kThreads, Smem::total),
                        "decode occupancy"))
            return -1;
        g_grid[dev] = sms * std::max(per_sm, 0);
        g_attr_set[dev] = true;
    }
    const int grid = g_grid[dev];
    if (grid < 1) return 0;

    // scratch: the barrier words (zeroed, self-resetting), then the down-phase sets of h
    const size_t sync_b = 256;
    const size_t sets_b = (size_t)a.n_tokens * a.n_used * p.dn.set_stride;
    if (sync_b > g_ds.counter_cap || sets_b > g_ds.partial_cap) {
        const size_t ccap = std::max(sync_b, g_ds.counter_cap), pcap = std::max(sets_b, g_ds.partial_cap);
        if (g_ds.mem) {
            cudaDeviceSynchronize();   // no kernel of an earlier call may still use it
            cudaFree(g_ds.mem);
        }
        g_ds = DecodeScratch{};
        if (!sb_cuda_ok(cudaMalloc(&g_ds.mem, ccap + pcap), "decode scratch")) return -1;
        if (!sb_cuda_ok(cudaMemset(g_ds.mem, 0, ccap), "decode scratch reset")) return -1;
        g_ds.counter_cap = ccap;
        g_ds.partial_cap = pcap;
    }
    if (g_ds.stale) {
        if (!sb_cuda_ok(cudaMemsetAsync(g_ds.mem, 0, g_ds.counter_cap, st), "decode scratch reset")) return -1;
        g_ds.stale = false;
    }
    uint8_t* b = (uint8_t*)g_ds.mem;
    p.sync = (unsigned*)b;
    p.hsets = b + g_ds.counter_cap;

    p.n_layers = a.n_layers;
    p.n_tokens = a.n_tokens;
    p.n_used = a.n_used;
    p.n_experts = a.n_experts;
    p.d_model = a.d_model;
    p.ff = a.ff;
    p.gu_stride = a.gu_expert_stride;
    p.dn_stride = a.down_expert_stride;
    p.x = a.x;
    p.out = a.out;
    p.accumulate = a.accumulate;
    p.xrows = a.xrows;
    p.n_xrows = a.n_xrows;
    p.h = a.h;
    p.err = a.err;
    const size_t per_layer = (size_t)a.n_tokens * a.n_used;
    for (int L = 0; L < a.n_layers; ++L) {
        p.layer[L].gate = (const uint8_t*)a.gate_banks[L];
        p.layer[L].up = (const uint8_t*)a.up_banks[L];
        p.layer[L].down = (const uint8_t*)a.down_banks[L];
        p.layer[L].ids = a.ids + L * per_layer;
        p.layer[L].w = a.w + L * per_layer;
    }

    const int tslot = sb_timing_begin("decode_iq3s", st);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Smem::total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, k_decode_iq3s, p);
    sb_timing_end(tslot, st);
    return sb_cuda_ok(e, "decode launch") ? 1 : -1;
}
